"""Public API of the synthetic package in the reference's calling forms (sae_lens/synthetic):
the activation iterator, train_toy_sae with snapshots, the eval result and scaler, the stats
functions, the feature ordering helpers, the plot's data and SyntheticModel.to."""

from __future__ import annotations

import pytest
import torch

from saelens_b200.models.standard import StandardTrainingSAE, StandardTrainingSAEConfig
from saelens_b200.synthetic import (
    ActivationGenerator,
    FeatureDictionary,
    LowRankCorrelationMatrix,
    SyntheticActivationIterator,
    SyntheticModel,
    SyntheticModelConfig,
    compute_correlation_matrix_stats,
    compute_low_rank_correlation_matrix_stats,
    compute_superposition_stats,
    eval_sae_on_synthetic_data,
    find_best_feature_ordering,
    find_best_feature_ordering_across_saes,
    generate_random_low_rank_correlation_matrix,
    init_sae_to_match_feature_dict,
    train_toy_sae,
)
from saelens_b200.synthetic.runner import feature_similarity_matrices
from saelens_b200.training.activation_scaler import ActivationScaler


def _setup(n=16, d=32, seed=0):
    torch.manual_seed(seed)
    fd = FeatureDictionary(n, d, seed=seed)
    gen = ActivationGenerator(n, 0.2, std_firing_magnitudes=0.1, mean_firing_magnitudes=1.0)
    return fd, gen


def _sae(n=16, d=32):
    return StandardTrainingSAE(StandardTrainingSAEConfig(d_in=d, d_sae=n, l1_coefficient=1e-3))


def test_iterator_reference_and_model_forms() -> None:
    fd, gen = _setup()
    it = SyntheticActivationIterator(fd, gen, 8)
    x = next(it)
    assert x.shape == (8, 32) and it.next_batch().shape == (8, 32)
    model = SyntheticModel(SyntheticModelConfig(num_features=16, hidden_dim=32, seed=1))
    it2 = SyntheticActivationIterator(model, 4, dtype=torch.float64)
    y = next(iter(it2))
    assert y.shape == (4, 32) and y.dtype == torch.float64
    with pytest.raises(TypeError):
        SyntheticActivationIterator(fd, gen)


def test_train_toy_sae_trains_and_takes_snapshots() -> None:
    fd, gen = _setup()
    sae = _sae()
    before = sae.W_dec.detach().clone()
    steps: list[int] = []
    train_toy_sae(sae, fd, gen, training_samples=64 * 20, batch_size=64, lr=1e-2, n_snapshots=3,
                  snapshot_fn=lambda trainer: steps.append(trainer.n_training_steps))
    assert not torch.equal(before, sae.W_dec.detach())
    assert len(steps) == 3 and steps == sorted(steps)
    with pytest.raises(ValueError):
        train_toy_sae(_sae(), fd, gen, training_samples=64, batch_size=64, n_snapshots=1)


def test_train_toy_sae_accepts_a_synthetic_model() -> None:
    model = SyntheticModel(SyntheticModelConfig(num_features=16, hidden_dim=32, seed=2))
    sae = _sae()
    before = sae.W_dec.detach().clone()
    train_toy_sae(sae, model, training_samples=32 * 5, batch_size=32)
    assert not torch.equal(before, sae.W_dec.detach())


def test_eval_reports_true_and_sae_l0_and_uses_the_scaler() -> None:
    fd, gen = _setup()
    sae = _sae()
    init_sae_to_match_feature_dict(sae, fd)
    torch.manual_seed(3)
    r = eval_sae_on_synthetic_data(sae, fd, gen, num_samples=2000, batch_size=500)
    assert r.true_l0 == pytest.approx(16 * 0.2, rel=0.1)
    assert r.sae_l0 > 0 and 0 <= r.dead_latents <= 16
    torch.manual_seed(3)
    unit = eval_sae_on_synthetic_data(sae, fd, gen, num_samples=2000, batch_size=500,
                                      activation_scaler=ActivationScaler(1.0))
    assert unit.explained_variance == pytest.approx(r.explained_variance, rel=1e-5)
    torch.manual_seed(3)
    scaled = eval_sae_on_synthetic_data(sae, fd, gen, num_samples=2000, batch_size=500,
                                        activation_scaler=ActivationScaler(3.0))
    assert scaled.true_l0 == pytest.approx(r.true_l0)
    assert scaled.sae_l0 != r.sae_l0 or scaled.explained_variance != r.explained_variance


def test_superposition_stats_of_orthogonal_and_overlapping_dictionaries() -> None:
    st = compute_superposition_stats(torch.eye(4), percentiles=[50])
    assert st.mean_max_abs_cos_sim == 0.0 and st.mean_percentile_abs_cos_sim[50] == 0.0
    assert st.num_features == 4 and st.hidden_dim == 4
    v = torch.tensor([[1.0, 0.0], [1.0, 1.0], [0.0, 1.0]])
    st = compute_superposition_stats(v, batch_size=2)
    c = 2 ** -0.5
    assert torch.allclose(st.max_abs_cos_sims, torch.tensor([c, c, c]), atol=1e-6)
    assert st.mean_abs_cos_sim == pytest.approx((c + 0 + c) / 3, abs=1e-6)
    fd, _ = _setup()
    assert compute_superposition_stats(fd).num_features == 16
    with pytest.raises(ValueError):
        compute_superposition_stats(torch.ones(1, 3))


def test_correlation_stats_dense_and_low_rank_agree() -> None:
    c = torch.tensor([[1.0, 0.5, -0.2], [0.5, 1.0, 0.0], [-0.2, 0.0, 1.0]])
    st = compute_correlation_matrix_stats(c)
    off = torch.tensor([0.5, -0.2, 0.5, 0.0, -0.2, 0.0])
    assert st.mean_correlation == pytest.approx(float(off.mean()))
    assert st.rms_correlation == pytest.approx(float(off.square().mean().sqrt()))
    lr = generate_random_low_rank_correlation_matrix(30, rank=3, correlation_scale=0.3, seed=0)
    dense = lr.correlation_factor @ lr.correlation_factor.T + torch.diag(lr.correlation_diag)
    a, b = compute_low_rank_correlation_matrix_stats(lr), compute_correlation_matrix_stats(dense)
    assert a.rms_correlation == pytest.approx(b.rms_correlation, rel=1e-5)
    assert a.mean_correlation == pytest.approx(b.mean_correlation, abs=1e-6)
    assert isinstance(lr, LowRankCorrelationMatrix) and a.num_features == 30


def test_feature_ordering_sorts_latents_by_their_best_true_feature() -> None:
    true = torch.eye(3)
    sae_feats = torch.tensor([[0.0, 0.0, 1.0], [1.0, 0.1, 0.0], [0.0, 1.0, 0.0]])
    order = find_best_feature_ordering(sae_feats, true)
    assert order.tolist() == [1, 2, 0]

    class _S:
        def __init__(self, w: torch.Tensor):
            self.W_dec = w

    class _F:
        feature_vectors = true

    good, bad = _S(sae_feats), _S(torch.ones(3, 3))
    assert find_best_feature_ordering_across_saes([bad, good], _F()).tolist() == [1, 2, 0]


def test_plot_data_reorders_rows_and_rounds() -> None:
    fd, _ = _setup()
    sae = _sae()
    init_sae_to_match_feature_dict(sae, fd, feature_ordering=torch.arange(15, -1, -1))
    enc, dec = feature_similarity_matrices(sae, fd, reorder_features=True)
    assert enc.shape == dec.shape == (16, 16)
    assert torch.allclose(dec.diagonal(), torch.ones(16), atol=0.011)
    assert torch.equal(dec, torch.round(dec * 100) / 100)
    _, plain = feature_similarity_matrices(sae, fd)
    assert torch.allclose(plain.flip(0).diagonal(), torch.ones(16), atol=0.011)


def test_synthetic_model_to_moves_the_generator_state() -> None:
    model = SyntheticModel(SyntheticModelConfig(num_features=8, hidden_dim=16, seed=4))
    assert model.to("cpu") is model
    assert model.to(None) is model
    assert model.activation_generator.firing_probabilities.device.type == "cpu"
    assert model.sample(5).shape == (5, 16)


def test_synthetic_model_from_prebuilt_components() -> None:
    cfg = SyntheticModelConfig(num_features=8, hidden_dim=16, seed=5)
    fd, gen = _setup(8, 16, seed=6)
    lr = generate_random_low_rank_correlation_matrix(8, rank=2, correlation_scale=0.2, seed=1)
    m = SyntheticModel(cfg, feature_dict=fd, activation_generator=gen, correlation_matrix=lr)
    assert m.feature_dict is fd and m.activation_generator is gen
    assert torch.equal(m.correlation.correlation_factor, lr.correlation_factor)
    h, f = m.sample_with_features(12)
    assert h.shape == (12, 16) and f.shape == (12, 8)
