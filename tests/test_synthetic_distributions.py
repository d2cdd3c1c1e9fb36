"""Firing-probability, magnitude and correlation generators of the synthetic package
(behaviour of sae_lens/synthetic/firing_probabilities.py, firing_magnitudes.py, correlation.py,
registry.py): shapes, ranges, orderings, seeding, validation, serialisation in the reference's
format, and the registry's two calling forms."""

from __future__ import annotations

from dataclasses import dataclass

import pytest
import torch

from saelens_b200.synthetic import (
    ConstantFiringProbabilityConfig,
    ConstantMagnitudeConfig,
    ExponentialMagnitudeConfig,
    FiringProbabilityConfig,
    FoldedNormalMagnitudeConfig,
    LinearFiringProbabilityConfig,
    LinearMagnitudeConfig,
    MagnitudeConfig,
    RandomFiringProbabilityConfig,
    ZipfianFiringProbabilityConfig,
    create_correlation_matrix_from_correlations,
    generate_magnitudes,
    generate_random_correlation_matrix,
    generate_random_correlations,
    generate_random_low_rank_correlation_matrix,
    get_firing_probability_class,
    get_magnitude_class,
    linear_firing_probabilities,
    random_firing_probabilities,
    register_firing_probability,
    register_magnitude,
    zipfian_firing_probabilities,
)
from saelens_b200.synthetic.distributions import correlation_thresholds


# ------------------------------------------------------------------ firing probabilities
@pytest.mark.parametrize("exponent", [0.5, 1.0, 2.0])
def test_zipfian_spans_the_range_in_descending_order(exponent: float) -> None:
    p = zipfian_firing_probabilities(100, exponent=exponent, max_prob=0.4, min_prob=0.02)
    assert p.shape == (100,)
    assert float(p[0]) == pytest.approx(0.4) and float(p[-1]) == pytest.approx(0.02)
    assert bool((p[1:] <= p[:-1]).all())


def test_zipfian_is_steeper_for_larger_exponents() -> None:
    a = zipfian_firing_probabilities(50, exponent=0.5)
    b = zipfian_firing_probabilities(50, exponent=2.0)
    assert float(b[5]) < float(a[5])  # most of the mass drops off earlier


@pytest.mark.parametrize("kw", [dict(exponent=0.0), dict(min_prob=0.0), dict(min_prob=0.5, max_prob=0.4),
                                dict(max_prob=1.5)])
def test_zipfian_rejects_bad_parameters(kw) -> None:
    with pytest.raises(ValueError):
        zipfian_firing_probabilities(10, **kw)
    with pytest.raises(ValueError):
        zipfian_firing_probabilities(0)


def test_single_feature_gets_the_maximum() -> None:
    assert zipfian_firing_probabilities(1, max_prob=0.3).tolist() == pytest.approx([0.3])
    assert linear_firing_probabilities(1, max_prob=0.2).tolist() == pytest.approx([0.2])


def test_linear_probabilities_decay_evenly() -> None:
    p = linear_firing_probabilities(11, max_prob=0.3, min_prob=0.1)
    assert float(p[0]) == pytest.approx(0.3) and float(p[-1]) == pytest.approx(0.1)
    steps = p[:-1] - p[1:]
    assert torch.allclose(steps, torch.full_like(steps, 0.02), atol=1e-6)
    assert torch.equal(linear_firing_probabilities(4, 0.2, 0.2), torch.full((4,), 0.2))
    with pytest.raises(ValueError):
        linear_firing_probabilities(4, max_prob=0.1, min_prob=0.2)


def test_random_probabilities_are_in_range_and_seeded() -> None:
    a = random_firing_probabilities(1000, max_prob=0.5, min_prob=0.1, seed=3)
    b = random_firing_probabilities(1000, max_prob=0.5, min_prob=0.1, seed=3)
    c = random_firing_probabilities(1000, max_prob=0.5, min_prob=0.1, seed=4)
    assert torch.equal(a, b) and not torch.equal(a, c)
    assert float(a.min()) >= 0.1 and float(a.max()) <= 0.5
    assert abs(float(a.mean()) - 0.3) < 0.02
    with pytest.raises(ValueError):
        random_firing_probabilities(10, max_prob=0.1, min_prob=0.1)


@pytest.mark.parametrize("cfg", [ZipfianFiringProbabilityConfig(exponent=1.5, max_prob=0.2, min_prob=0.01),
                                 LinearFiringProbabilityConfig(max_prob=0.3, min_prob=0.05),
                                 RandomFiringProbabilityConfig(max_prob=0.4, min_prob=0.1),
                                 ConstantFiringProbabilityConfig(probability=0.07)])
def test_probability_configs_generate_and_round_trip(cfg: FiringProbabilityConfig) -> None:
    p = cfg.generate(64, seed=0)
    assert p.shape == (64,) and float(p.min()) > 0 and float(p.max()) <= 1
    d = cfg.to_dict()
    assert d["generator_name"] == cfg.generator_name()
    back = FiringProbabilityConfig.from_dict(d)
    assert back == cfg and torch.equal(back.generate(64, seed=0), p)
    assert get_firing_probability_class(cfg.generator_name()) is type(cfg)


def test_probability_config_from_a_reference_style_dict() -> None:
    cfg = FiringProbabilityConfig.from_dict({"generator_name": "linear", "max_prob": 0.25, "min_prob": 0.05})
    assert isinstance(cfg, LinearFiringProbabilityConfig) and cfg.max_prob == 0.25
    with pytest.raises(ValueError):
        FiringProbabilityConfig.from_dict({"max_prob": 0.25})
    with pytest.raises(ValueError):
        get_firing_probability_class("no_such_generator")


def test_registry_accepts_name_and_class_or_decorator_and_refuses_a_second_class() -> None:
    @dataclass
    class HalfConfig(FiringProbabilityConfig):
        @classmethod
        def generator_name(cls) -> str:
            return "test_half"

        def generate(self, num_features: int, seed: int | None = None) -> torch.Tensor:
            return torch.full((num_features,), 0.5)

    register_firing_probability("test_half", HalfConfig)
    register_firing_probability("test_half", HalfConfig)  # the same class again is harmless
    assert get_firing_probability_class("test_half") is HalfConfig
    assert isinstance(FiringProbabilityConfig.from_dict({"generator_name": "test_half"}), HalfConfig)

    @dataclass
    class Other(HalfConfig):
        pass

    with pytest.raises(ValueError, match="already registered"):
        register_firing_probability("test_half", Other)

    @register_magnitude
    @dataclass
    class TwoConfig(MagnitudeConfig):
        @classmethod
        def generator_name(cls) -> str:
            return "test_two"

        def generate(self, num_features: int, seed: int | None = None) -> torch.Tensor:
            return torch.full((num_features,), 2.0)

    assert get_magnitude_class("test_two") is TwoConfig
    assert torch.equal(generate_magnitudes(3, TwoConfig()), torch.full((3,), 2.0))


# ------------------------------------------------------------------ magnitudes
def test_magnitude_generators() -> None:
    assert torch.equal(generate_magnitudes(4, 2.5), torch.full((4,), 2.5))
    assert torch.equal(ConstantMagnitudeConfig(value=3.0).generate(2), torch.full((2,), 3.0))
    lin = LinearMagnitudeConfig(start=1.0, end=3.0).generate(5)
    assert torch.allclose(lin, torch.tensor([1.0, 1.5, 2.0, 2.5, 3.0]))
    exp = ExponentialMagnitudeConfig(start=1.0, end=16.0).generate(5)
    assert torch.allclose(exp, torch.tensor([1.0, 2.0, 4.0, 8.0, 16.0]), rtol=1e-5)
    ratios = exp[1:] / exp[:-1]
    assert torch.allclose(ratios, torch.full_like(ratios, 2.0), rtol=1e-5)
    assert LinearMagnitudeConfig(start=2.0, end=5.0).generate(1).tolist() == [2.0]


def test_folded_normal_magnitudes_are_non_negative_seeded_and_clamped() -> None:
    cfg = FoldedNormalMagnitudeConfig(mean=0.0, std=1.0)
    a, b = cfg.generate(5000, seed=1), cfg.generate(5000, seed=1)
    assert torch.equal(a, b) and bool((a >= 0).all())
    assert abs(float(a.mean()) - (2 / torch.pi) ** 0.5) < 0.05  # E|N(0,1)| = sqrt(2/pi)
    c = FoldedNormalMagnitudeConfig(mean=1.0, std=2.0, min_value=0.5, max_value=2.0).generate(2000, seed=2)
    assert float(c.min()) >= 0.5 and float(c.max()) <= 2.0


@pytest.mark.parametrize("make", [lambda: LinearMagnitudeConfig(start=0.0, end=1.0),
                                  lambda: ExponentialMagnitudeConfig(start=1.0, end=-1.0),
                                  lambda: FoldedNormalMagnitudeConfig(std=0.0),
                                  lambda: FoldedNormalMagnitudeConfig(min_value=-1.0),
                                  lambda: FoldedNormalMagnitudeConfig(min_value=2.0, max_value=1.0)])
def test_magnitude_configs_reject_bad_parameters(make) -> None:
    with pytest.raises(ValueError):
        make()


def test_magnitude_config_round_trip() -> None:
    for cfg in (ConstantMagnitudeConfig(value=2.0), LinearMagnitudeConfig(start=1.0, end=2.0),
                ExponentialMagnitudeConfig(start=0.5, end=4.0), FoldedNormalMagnitudeConfig(mean=1.0, std=0.5)):
        d = cfg.to_dict()
        assert d["generator_name"] == cfg.generator_name()
        assert MagnitudeConfig.from_dict(d) == cfg
    # the key this package wrote before also loads
    assert MagnitudeConfig.from_dict({"generator": "constant", "value": 4.0}) == ConstantMagnitudeConfig(value=4.0)


# ------------------------------------------------------------------ correlations
def test_random_correlations_respect_ratios_and_strengths() -> None:
    n = 60
    corr = generate_random_correlations(n, positive_ratio=0.7, uncorrelated_ratio=0.4,
                                        min_correlation_strength=0.2, max_correlation_strength=0.5, seed=0)
    pairs = n * (n - 1) // 2
    assert all(i < j for i, j in corr)
    assert abs(len(corr) / pairs - 0.6) < 0.05
    vals = torch.tensor(list(corr.values()))
    assert float(vals.abs().min()) >= 0.2 and float(vals.abs().max()) <= 0.5
    assert abs(float((vals > 0).float().mean()) - 0.7) < 0.05
    assert corr == generate_random_correlations(n, positive_ratio=0.7, uncorrelated_ratio=0.4,
                                                min_correlation_strength=0.2, max_correlation_strength=0.5,
                                                seed=0)


@pytest.mark.parametrize("kw", [dict(positive_ratio=1.5), dict(uncorrelated_ratio=-0.1),
                                dict(min_correlation_strength=0.6, max_correlation_strength=0.5),
                                dict(max_correlation_strength=1.2)])
def test_correlation_parameters_are_validated(kw) -> None:
    with pytest.raises(ValueError):
        generate_random_correlations(5, **kw)
    with pytest.raises(ValueError):
        generate_random_correlation_matrix(5, **kw)


@pytest.mark.parametrize("n", [1, 2, 30])
def test_random_correlation_matrix_is_a_correlation_matrix(n: int) -> None:
    m = generate_random_correlation_matrix(n, max_correlation_strength=0.9, seed=5, dtype="float64")
    assert m.shape == (n, n) and m.dtype == torch.float64
    assert torch.allclose(m, m.T)
    assert torch.allclose(m.diagonal(), torch.ones(n, dtype=torch.float64), atol=1e-6)
    assert float(torch.linalg.eigvalsh(m).min()) > -1e-6


def test_correlations_to_a_matrix_and_repair_of_impossible_sets() -> None:
    m = create_correlation_matrix_from_correlations(3, {(0, 1): 0.5})
    assert float(m[0, 1]) == pytest.approx(0.5) and float(m[1, 0]) == pytest.approx(0.5)
    assert float(m[0, 2]) == 0.0 and float(m[2, 2]) == 1.0
    # three mutually strongly anti-correlated features are impossible: the result is repaired
    bad = create_correlation_matrix_from_correlations(3, {(0, 1): -0.9, (0, 2): -0.9, (1, 2): -0.9})
    assert float(torch.linalg.eigvalsh(bad.double()).min()) > -1e-6
    assert torch.allclose(bad.diagonal(), torch.ones(3), atol=1e-5)


def test_low_rank_correlation_has_a_unit_diagonal() -> None:
    lr = generate_random_low_rank_correlation_matrix(200, rank=4, correlation_scale=0.3, seed=1)
    f, d = lr
    assert f.shape == (200, 4) and d.shape == (200,)
    assert torch.allclose(f.square().sum(1) + d, torch.ones(200), atol=1e-5)
    assert bool((d > 0).all())
    big = generate_random_low_rank_correlation_matrix(50, rank=3, correlation_scale=2.0, seed=1)
    assert bool((big.correlation_diag > 0).all())  # rows shrunk below unit norm
    with pytest.raises(ValueError):
        generate_random_low_rank_correlation_matrix(10, rank=0)


def test_copula_thresholds_give_the_marginal_rates() -> None:
    p = torch.tensor([0.01, 0.1, 0.5, 0.9])
    t = correlation_thresholds(p)
    upper = 0.5 * torch.erfc(t / 2 ** 0.5)  # P(N(0,1) > t)
    assert torch.allclose(upper, p, atol=1e-6)
