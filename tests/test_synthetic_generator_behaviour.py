"""Statistical behaviour of the synthetic activation generator (sae_lens/synthetic/
activation_generator.py): firing rates, magnitudes, non-negativity, modifier chaining,
correlated firing (full and low-rank) and its validation.  Rates are checked against their
binomial standard error, magnitudes against the sampling error of their mean and spread."""

from __future__ import annotations

import math

import pytest
import torch

from saelens_b200.synthetic import ActivationGenerator, LowRankCorrelationMatrix
from saelens_b200.synthetic.distributions import generate_random_correlation_matrix


def _dense(x: torch.Tensor) -> torch.Tensor:
    return x.to_dense() if x.is_sparse else x


def _within_binomial(rate: torch.Tensor, p: torch.Tensor, n: int, z: float = 5.0) -> bool:
    se = (p * (1 - p) / n).sqrt().clamp_min(1e-4)
    return bool(((rate - p).abs() <= z * se).all())


@pytest.mark.parametrize("sparse", [False, True])
def test_firing_rates_follow_the_probabilities(sparse: bool) -> None:
    torch.manual_seed(0)
    p = torch.tensor([0.0, 0.02, 0.1, 0.3, 0.7, 1.0])
    gen = ActivationGenerator(6, p, use_sparse_tensors=sparse)
    n = 20000
    x = _dense(gen.sample(n))
    rate = (x > 0).float().mean(0)
    assert _within_binomial(rate, p, n)
    assert float(rate[0]) == 0.0 and float(rate[-1]) == 1.0


@pytest.mark.parametrize("sparse", [False, True])
def test_magnitudes_follow_mean_and_spread(sparse: bool) -> None:
    torch.manual_seed(1)
    mean = torch.tensor([2.0, 5.0, 10.0])
    std = torch.tensor([0.1, 0.5, 1.0])
    gen = ActivationGenerator(3, 0.5, std_firing_magnitudes=std, mean_firing_magnitudes=mean,
                              use_sparse_tensors=sparse)
    x = _dense(gen.sample(20000))
    for j in range(3):
        v = x[:, j][x[:, j] > 0]
        assert abs(float(v.mean()) - float(mean[j])) <= 5 * float(std[j]) / math.sqrt(v.numel())
        assert abs(float(v.std()) - float(std[j])) <= 0.05 * float(std[j]) + 1e-3


@pytest.mark.parametrize("sparse", [False, True])
def test_activations_are_never_negative(sparse: bool) -> None:
    torch.manual_seed(2)
    gen = ActivationGenerator(8, 0.5, std_firing_magnitudes=3.0, mean_firing_magnitudes=0.5,
                              use_sparse_tensors=sparse)
    x = _dense(gen.sample(5000))
    assert bool((x >= 0).all())
    assert float((x == 0).float().mean()) > 0.5  # the clipped tail adds zeros to the non-firing half


def test_scalar_and_tensor_parameters_and_string_dtype() -> None:
    gen = ActivationGenerator(4, 0.25, std_firing_magnitudes=0.0, mean_firing_magnitudes=torch.tensor(3.0),
                              dtype="float64")
    assert gen.firing_probabilities.shape == (4,) and gen.firing_probabilities.dtype == torch.float64
    assert torch.equal(gen.mean_firing_magnitudes, torch.full((4,), 3.0, dtype=torch.float64))
    x = gen.sample(100)
    assert x.dtype == torch.float64 and set(x.unique().tolist()) <= {0.0, 3.0}
    with pytest.raises(ValueError):
        ActivationGenerator(4, torch.tensor([0.1, 0.2, 0.3]))
    with pytest.raises(ValueError):
        ActivationGenerator(2, torch.tensor([0.5, 1.5]))


def test_forward_is_sample() -> None:
    gen = ActivationGenerator(16, 0.2, std_firing_magnitudes=0.3)
    torch.manual_seed(3)
    a = gen(64)
    torch.manual_seed(3)
    b = gen.sample(64)
    assert torch.equal(a, b)


def test_modifiers_chain_in_order_and_the_result_is_clipped() -> None:
    torch.manual_seed(4)
    calls: list[str] = []

    def double(x: torch.Tensor) -> torch.Tensor:
        calls.append("double")
        return x * 2

    def shift(x: torch.Tensor, generator: ActivationGenerator) -> torch.Tensor:
        calls.append("shift")
        assert isinstance(generator, ActivationGenerator)
        return x - 3.0

    gen = ActivationGenerator(4, 1.0, mean_firing_magnitudes=1.0, modify_activations=[double, shift])
    x = gen.sample(10)
    assert calls == ["double", "shift"]
    assert bool((x == 0).all())  # 1 * 2 - 3 < 0, clipped by the final ReLU

    gen = ActivationGenerator(4, 1.0, mean_firing_magnitudes=2.0, modify_activations=double)
    assert bool((gen.sample(5) == 4.0).all())
    assert ActivationGenerator(4, 1.0, modify_activations=[]).modify_activations is None


def test_a_type_error_inside_a_two_argument_modifier_is_not_swallowed() -> None:
    def broken(x: torch.Tensor, generator: ActivationGenerator) -> torch.Tensor:
        raise TypeError("inside the modifier")

    gen = ActivationGenerator(4, 1.0, modify_activations=broken)
    with pytest.raises(TypeError, match="inside the modifier"):
        gen.sample(3)


def test_modifier_on_sparse_samples_keeps_them_sparse_and_clipped() -> None:
    torch.manual_seed(5)

    def negate_first(x: torch.Tensor) -> torch.Tensor:
        d = x.to_dense()
        d[:, 0] = -d[:, 0]
        return d.to_sparse()

    gen = ActivationGenerator(3, 1.0, mean_firing_magnitudes=1.0, modify_activations=negate_first,
                              use_sparse_tensors=True)
    x = gen.sample(7)
    assert x.is_sparse
    d = x.to_dense()
    assert bool((d[:, 0] == 0).all()) and bool((d[:, 1:] == 1.0).all())


def test_full_correlation_keeps_marginals_and_correlates_firing() -> None:
    torch.manual_seed(6)
    p = torch.tensor([0.2, 0.2, 0.3, 0.1])
    c = torch.eye(4)
    c[0, 1] = c[1, 0] = 0.8
    c[2, 3] = c[3, 2] = -0.5
    gen = ActivationGenerator(4, p, correlation_matrix=c)
    n = 40000
    fired = (gen.sample(n) > 0).float()
    assert _within_binomial(fired.mean(0), p, n)
    r = torch.corrcoef(fired.T)
    assert float(r[0, 1]) > 0.4
    assert float(r[2, 3]) < -0.05
    assert abs(float(r[0, 2])) < 0.03


def test_low_rank_correlation_keeps_marginals() -> None:
    torch.manual_seed(7)
    n_feat = 32
    p = torch.linspace(0.02, 0.4, n_feat)
    factor = torch.randn(n_feat, 3) * 0.3
    diag = 1.0 - (factor ** 2).sum(1)
    gen = ActivationGenerator(n_feat, p, correlation_matrix=LowRankCorrelationMatrix(factor, diag))
    n = 30000
    rate = (gen.sample(n) > 0).float().mean(0)
    assert _within_binomial(rate, p, n)
    # the plain (factor, diag) tuple is accepted as well
    ActivationGenerator(n_feat, p, correlation_matrix=(factor, diag))


def test_generated_correlation_matrix_is_a_valid_input() -> None:
    c = generate_random_correlation_matrix(16, seed=3)
    assert torch.allclose(c, c.T) and torch.allclose(c.diagonal(), torch.ones(16))
    assert float(torch.linalg.eigvalsh(c.double()).min()) > 0
    ActivationGenerator(16, 0.1, correlation_matrix=c)


@pytest.mark.parametrize("bad", ["shape", "diag", "asym", "not_pd"])
def test_invalid_correlation_matrices_are_rejected(bad: str) -> None:
    c = torch.eye(3)
    if bad == "shape":
        c = torch.eye(4)
    elif bad == "diag":
        c[1, 1] = 0.5
    elif bad == "asym":
        c[0, 1] = 0.3
    else:  # unit diagonal, symmetric, but an eigenvalue below zero
        c = torch.tensor([[1.0, 0.9, -0.9], [0.9, 1.0, 0.9], [-0.9, 0.9, 1.0]])
    with pytest.raises(ValueError):
        ActivationGenerator(3, 0.1, correlation_matrix=c)


@pytest.mark.parametrize("bad", ["factor_rows", "diag_shape", "diag_zero", "diag_negative"])
def test_invalid_low_rank_correlations_are_rejected(bad: str) -> None:
    factor, diag = torch.randn(5, 2) * 0.1, torch.full((5,), 0.9)
    if bad == "factor_rows":
        factor = torch.randn(4, 2)
    elif bad == "diag_shape":
        diag = torch.full((4,), 0.9)
    elif bad == "diag_zero":
        diag[2] = 0.0
    else:
        diag[0] = -0.1
    with pytest.raises(ValueError):
        ActivationGenerator(5, 0.1, correlation_matrix=(factor, diag))
