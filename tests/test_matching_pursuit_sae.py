"""Matching-pursuit SAE (behaviour of sae_lens/saes/matching_pursuit_sae.py; cases follow
tests/saes/test_matching_pursuit_sae.py)."""

import pytest
import torch

from saelens_b200.models.matching_pursuit import (
    MatchingPursuitSAE,
    MatchingPursuitSAEConfig,
    MatchingPursuitTrainingSAE,
    MatchingPursuitTrainingSAEConfig,
    _encode_matching_pursuit,
)
from saelens_b200.models.sae import SAE, TrainStepInput


def _orthogonal(sae, seed=0):
    torch.manual_seed(seed)
    with torch.no_grad():
        torch.nn.init.orthogonal_(sae.W_dec)
        sae.b_dec.copy_(torch.randn_like(sae.b_dec))
    feats = (torch.randn(32, 10) - 0.25).relu()
    return feats, feats @ sae.W_dec + sae.b_dec


@pytest.mark.parametrize("training", [False, True])
def test_recovers_features_of_an_orthogonal_dictionary(training):
    sae = (MatchingPursuitTrainingSAE(MatchingPursuitTrainingSAEConfig(d_in=10, d_sae=10, residual_threshold=1e-8))
           if training else MatchingPursuitSAE(MatchingPursuitSAEConfig(d_in=10, d_sae=10, residual_threshold=1e-8)))
    true, x = _orthogonal(sae)
    with torch.no_grad():
        f = sae.encode(x)
        torch.testing.assert_close(f, true, rtol=1e-4, atol=1e-5)
        torch.testing.assert_close(sae.decode(f), x, rtol=1e-4, atol=1e-5)


@pytest.mark.parametrize("training", [False, True])
def test_max_iterations_is_respected(training):
    kw = dict(d_in=10, d_sae=10, residual_threshold=1e-8, max_iterations=2)
    sae = (MatchingPursuitTrainingSAE(MatchingPursuitTrainingSAEConfig(**kw)) if training
           else MatchingPursuitSAE(MatchingPursuitSAEConfig(**kw)))
    true, x = _orthogonal(sae)
    with torch.no_grad():
        f = sae.encode(x)
    assert int((f > 0).sum(-1).max()) == 2
    torch.testing.assert_close(f[f > 0], true[f > 0], rtol=1e-4, atol=1e-5)


def test_3d_inputs_match_flattened():
    sae = MatchingPursuitTrainingSAE(MatchingPursuitTrainingSAEConfig(d_in=10, d_sae=10, residual_threshold=1e-8))
    torch.manual_seed(0)
    x = torch.randn(8, 5, 10)
    with torch.no_grad():
        a, b = sae.encode(x), sae.encode(x.reshape(40, 10))
    assert a.shape == (8, 5, 10)
    torch.testing.assert_close(a.reshape(40, 10), b)


def test_decoder_init_norm_warning():
    with pytest.warns(UserWarning):
        MatchingPursuitTrainingSAEConfig(d_in=10, d_sae=10, decoder_init_norm=0.3)


def test_encode_matches_greedy_restatement():
    """Greedy pursuit: pick argmax relu(r . w_j), add the coefficient, subtract it from r."""
    torch.manual_seed(1)
    W = torch.randn(20, 10)
    W = W / W.norm(dim=1, keepdim=True)
    x = torch.randn(6, 10)
    got = _encode_matching_pursuit(x, W, residual_threshold=0.0, max_iterations=4, stop_on_duplicate_support=False)
    want = torch.zeros(6, 20)
    r = x.clone()
    for _ in range(4):
        c = torch.relu(r @ W.T)
        v, j = c.max(dim=-1)
        want[torch.arange(6), j] += v
        r = r - v[:, None] * W[j]
    torch.testing.assert_close(got, want, rtol=1e-5, atol=1e-6)
    assert int((got > 0).sum(-1).max()) <= 4


def test_training_metrics_only_on_logging_steps():
    torch.manual_seed(0)
    sae = MatchingPursuitTrainingSAE(MatchingPursuitTrainingSAEConfig(d_in=10, d_sae=20, residual_threshold=1e-2))
    x = torch.randn(8, 10)
    for logging in (True, False):
        out = sae.training_forward_pass(TrainStepInput(sae_in=x, coefficients={}, dead_neuron_mask=None,
                                                       n_training_steps=0, is_logging_step=logging))
        keys = {"max_l0", "min_l0", "residual_norm", "residual_threshold_converged_portion"}
        assert keys <= set(out.metrics) if logging else len(out.metrics) == 0


def test_export_roundtrip(tmp_path):
    torch.manual_seed(0)
    sae = MatchingPursuitTrainingSAE(MatchingPursuitTrainingSAEConfig(d_in=10, d_sae=20, residual_threshold=1e-3))
    sae.save_inference_model(tmp_path)
    inf = SAE.load_from_disk(tmp_path)
    assert isinstance(inf, MatchingPursuitSAE)
    x = torch.randn(5, 10)
    with torch.no_grad():
        torch.testing.assert_close(inf.encode(x), sae.encode(x))
