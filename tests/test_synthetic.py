"""Synthetic data package: distributions, generator statistics, hierarchy rules, model round trip,
metrics and a short runner training on CPU."""

import math

import pytest
import torch

from saelens_b200 import synthetic as S


def test_firing_probability_generators():
    z = S.zipfian_firing_probabilities(100, exponent=1.0, max_prob=0.3, min_prob=0.01)
    assert z[0].item() == pytest.approx(0.3) and z[-1].item() == pytest.approx(0.01)
    assert (z[:-1] >= z[1:]).all()
    lin = S.linear_firing_probabilities(5, 0.5, 0.1)
    assert torch.allclose(lin, torch.tensor([0.5, 0.4, 0.3, 0.2, 0.1]))
    r = S.random_firing_probabilities(1000, 0.4, 0.1, seed=3)
    assert r.min() >= 0.1 and r.max() <= 0.4
    assert torch.equal(r, S.random_firing_probabilities(1000, 0.4, 0.1, seed=3))
    cfg = S.ZipfianFiringProbabilityConfig(exponent=0.7)
    back = S.FiringProbabilityConfig.from_dict(cfg.to_dict())
    assert back == cfg and torch.allclose(back.generate(10), cfg.generate(10))
    with pytest.raises(ValueError):
        S.zipfian_firing_probabilities(10, max_prob=0.1, min_prob=0.2)


def test_magnitude_generators():
    e = S.ExponentialMagnitudeConfig(start=1.0, end=8.0).generate(4)
    assert torch.allclose(e, torch.tensor([1.0, 2.0, 4.0, 8.0]), rtol=1e-5)
    fn = S.FoldedNormalMagnitudeConfig(mean=0.0, std=1.0, max_value=2.0).generate(1000, seed=1)
    assert (fn >= 0).all() and (fn <= 2.0).all()
    assert S.MagnitudeConfig.from_dict(S.LinearMagnitudeConfig(1.0, 3.0).to_dict()) == S.LinearMagnitudeConfig(1.0, 3.0)
    assert torch.equal(S.generate_magnitudes(3, 2.5), torch.full((3,), 2.5))


def test_independent_firing_rates_and_magnitudes():
    p = torch.tensor([0.5, 0.1, 0.02, 0.0])
    gen = S.ActivationGenerator(4, p, std_firing_magnitudes=0.0, mean_firing_magnitudes=torch.tensor([1.0, 2.0, 3.0, 4.0]))
    torch.manual_seed(0)
    f = gen.sample(100_000)
    rate = (f > 0).float().mean(0)
    assert torch.allclose(rate, p, atol=5e-3)
    assert torch.allclose(f[:, 1][f[:, 1] > 0], torch.tensor(2.0))
    sp = S.ActivationGenerator(4, p, use_sparse_tensors=True).sample(1000)
    assert sp.is_sparse


def test_correlated_firing_keeps_marginals_and_correlates():
    corr = S.create_correlation_matrix_from_correlations(3, {(0, 1): 0.9}, default_correlation=0.0)
    gen = S.ActivationGenerator(3, torch.tensor([0.2, 0.2, 0.2]), correlation_matrix=corr)
    torch.manual_seed(0)
    fires = (gen.sample(50_000) > 0).float()
    assert torch.allclose(fires.mean(0), torch.full((3,), 0.2), atol=1e-2)
    c = torch.corrcoef(fires.T)
    assert c[0, 1] > 0.5 and abs(c[0, 2]) < 0.05
    lr = S.generate_random_low_rank_correlation_matrix(500, rank=8, correlation_scale=0.2, seed=0)
    full = lr.correlation_factor @ lr.correlation_factor.T + torch.diag(lr.correlation_diag)
    assert torch.allclose(full.diagonal(), torch.ones(500), atol=1e-5)
    gen2 = S.ActivationGenerator(500, 0.05, correlation_matrix=lr)
    assert abs((gen2.sample(20_000) > 0).float().mean().item() - 0.05) < 5e-3
    m = S.generate_random_correlation_matrix(20, seed=0)
    assert torch.linalg.eigvalsh(m.double()).min() > -1e-6 and torch.allclose(m.diagonal(), torch.ones(20))


def test_hierarchy_parent_gating_and_mutual_exclusion():
    tree = S.HierarchyNode(0, [S.HierarchyNode(1), S.HierarchyNode(2), S.HierarchyNode(3)],
                           mutually_exclusive_children=True)
    mod = S.hierarchy_modifier(tree)
    x = torch.tensor([[0.0, 1.0, 1.0, 0.0], [2.0, 1.0, 1.0, 1.0], [1.0, 0.0, 0.0, 0.0]])
    y = mod(x)
    assert torch.equal(y[0], torch.zeros(4))  # parent silent: children silenced
    assert y[1, 0] == 2.0 and int((y[1, 1:] > 0).sum()) == 1  # exactly one sibling survives
    assert torch.equal(y[2], x[2])
    h = S.generate_hierarchy(100, S.HierarchyConfig(total_root_nodes=3, branching_factor=(2, 3), max_depth=2,
                                                     mutually_exclusive_portion=1.0), seed=0)
    assert len(h.roots) == 3 and all(len(r.children) >= 2 for r in h.roots)
    assert S.Hierarchy.from_dict(h.to_dict()) == h
    p = torch.full((100,), 0.1)
    corr = h.compute_probability_correction_factors(p)
    child = h.roots[0].children[0].feature_index
    assert corr[h.roots[0].feature_index] == 1.0 and corr[child] > 1.0 / 0.1 - 1e-4


def test_synthetic_model_roundtrip(tmp_path):
    cfg = S.SyntheticModelConfig(num_features=64, hidden_dim=32, seed=1,
                                 correlation=S.LowRankCorrelationConfig(rank=4, correlation_scale=0.1),
                                 hierarchy=S.HierarchyConfig(total_root_nodes=2, branching_factor=3, max_depth=1),
                                 mean_firing_magnitude=S.LinearMagnitudeConfig(1.0, 2.0))
    m = S.SyntheticModel(cfg)
    fv = m.feature_dict.feature_vectors
    assert torch.allclose(fv.norm(dim=1), torch.ones(64), atol=1e-4)
    h, f = m.sample_with_features(16)
    assert h.shape == (16, 32) and f.shape == (16, 64)
    assert torch.allclose(h, f @ fv + m.feature_dict.bias, atol=1e-5)
    m.save(tmp_path / "m")
    m2 = S.SyntheticModel.load_from_disk(tmp_path / "m")
    assert torch.equal(m2.feature_dict.feature_vectors, fv.detach())
    assert torch.equal(m2.activation_generator.firing_probabilities, m.activation_generator.firing_probabilities)
    assert m2.hierarchy == m.hierarchy and m2.cfg.to_dict() == cfg.to_dict()


def test_metrics():
    gt = torch.eye(4)
    perm = gt[[2, 0, 3, 1]]
    assert S.mean_correlation_coefficient(perm, gt) == pytest.approx(1.0)
    assert S.feature_uniqueness(torch.cat([gt, gt[:1]]), gt) == pytest.approx(4 / 5)
    lat = torch.tensor([[1.0, 0, 0, 0], [0, 0, 0, 0]])
    acts = torch.tensor([[1.0, 0, 0, 0], [1.0, 0, 0, 0]])
    m = S.compute_classification_metrics(lat, acts, gt, gt)
    assert m.precision == pytest.approx(0.25) and m.recall == pytest.approx(0.125)
    ev = S.ExplainedVarianceCalculator(2)
    x = torch.randn(100, 2)
    ev.add_batch(x, x)
    assert ev.compute() == pytest.approx(1.0)
    st = S.compute_superposition_stats(torch.eye(3))
    assert st.mean_max_abs_cos_sim == 0.0 and st.mean_abs_cos_sim == 0.0 and st.num_features == 3


def test_runner_recovers_features_cpu(tmp_path):
    from saelens_b200.models.topk import TopKTrainingSAEConfig

    torch.manual_seed(0)
    cfg = S.SyntheticSAERunnerConfig(
        sae=TopKTrainingSAEConfig(d_in=32, d_sae=32, k=3, device="cpu"),
        synthetic_model=S.SyntheticModelConfig(num_features=32, hidden_dim=32, seed=0,
                                               firing_probability=S.ConstantFiringProbabilityConfig(0.06)),
        training_samples=256 * 120, train_batch_size_samples=256, lr=3e-3, eval_samples=4096, device="cpu",
        output_path=str(tmp_path / "out"))
    res = S.SyntheticSAERunner(cfg).run()
    assert res.eval_result.explained_variance > 0.5
    assert res.eval_result.mcc > 0.5
    assert (tmp_path / "out" / "eval_results.json").exists()
    cfg2 = S.SyntheticSAERunnerConfig.from_dict(cfg.to_dict())
    assert cfg2.sae.k == 3 and cfg2.training_samples == cfg.training_samples
    order = S.find_best_feature_ordering_from_sae(res.sae, res.synthetic_model.feature_dict)
    assert sorted(order.tolist()) == list(range(32))
