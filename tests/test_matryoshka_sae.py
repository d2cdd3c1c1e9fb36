"""Matryoshka BatchTopK (behaviour of sae_lens/saes/matryoshka_batchtopk_sae.py; cases follow
tests/saes/test_matryoshka_batchtopk_sae.py)."""

import pytest
import torch

from saelens_b200.models.batchtopk import (
    BatchTopKTrainingSAE,
    BatchTopKTrainingSAEConfig,
    MatryoshkaBatchTopKTrainingSAE,
    MatryoshkaBatchTopKTrainingSAEConfig,
)
from saelens_b200.models.sae import TrainStepInput
from saelens_b200.models.topk import calculate_topk_aux_acts


def _rand(sae, seed=0):
    torch.manual_seed(seed)
    with torch.no_grad():
        for p in sae.parameters():
            p.copy_(torch.randn_like(p) * 0.5)


def _step(x, dead=None):
    return TrainStepInput(sae_in=x, coefficients={}, dead_neuron_mask=dead, n_training_steps=0, is_logging_step=False)


def test_widths_validation():
    with pytest.warns(UserWarning, match="final matryoshka level"):
        s = MatryoshkaBatchTopKTrainingSAE(MatryoshkaBatchTopKTrainingSAEConfig(d_in=4, d_sae=8, k=2,
                                                                               matryoshka_widths=[2, 4]))
    assert s.cfg.matryoshka_widths == [2, 4, 8]
    s = MatryoshkaBatchTopKTrainingSAE(MatryoshkaBatchTopKTrainingSAEConfig(d_in=4, d_sae=8, k=2,
                                                                           matryoshka_widths=[2, 8]))
    assert s.cfg.matryoshka_widths == [2, 8]
    for bad in ([4, 4, 8], [6, 2, 8]):
        with pytest.raises(ValueError, match="strictly increasing"):
            MatryoshkaBatchTopKTrainingSAE(MatryoshkaBatchTopKTrainingSAEConfig(d_in=4, d_sae=8, k=2,
                                                                               matryoshka_widths=bad))


def test_inner_losses_are_prefix_reconstructions_added_to_the_loss():
    cfg = MatryoshkaBatchTopKTrainingSAEConfig(d_in=8, d_sae=12, k=3, matryoshka_widths=[4, 8, 12],
                                               rescale_acts_by_decoder_norm=False)
    sae = MatryoshkaBatchTopKTrainingSAE(cfg)
    _rand(sae)
    x = torch.randn(16, 8)
    with torch.no_grad():
        base_sae = BatchTopKTrainingSAE(BatchTopKTrainingSAEConfig(d_in=8, d_sae=12, k=3,
                                                                   rescale_acts_by_decoder_norm=False))
        base_sae.load_state_dict(sae.state_dict())
        base = base_sae.training_forward_pass(_step(x))
        out = sae.training_forward_pass(_step(x))
        f = out.feature_acts
        for w in (4, 8):
            want = ((f[:, :w] @ sae.W_dec[:w] + sae.b_dec - x) ** 2).sum(-1).mean()
            torch.testing.assert_close(out.losses[f"inner_mse_loss_{w}"], want)
        assert "inner_mse_loss_12" not in out.losses
        torch.testing.assert_close(out.loss, base.loss + out.losses["inner_mse_loss_4"] + out.losses["inner_mse_loss_8"])


def test_single_level_matches_batchtopk():
    with pytest.warns(UserWarning):
        m = MatryoshkaBatchTopKTrainingSAE(MatryoshkaBatchTopKTrainingSAEConfig(d_in=8, d_sae=12, k=3,
                                                                               matryoshka_widths=[12]))
    b = BatchTopKTrainingSAE(BatchTopKTrainingSAEConfig(d_in=8, d_sae=12, k=3))
    _rand(m)
    b.load_state_dict(m.state_dict())
    x = torch.randn(16, 8)
    with torch.no_grad():
        torch.testing.assert_close(m.training_forward_pass(_step(x)).loss, b.training_forward_pass(_step(x)).loss)


def test_matryoshka_aux_loss_manual():
    d_in, k_aux = 4, 2
    sae = MatryoshkaBatchTopKTrainingSAE(MatryoshkaBatchTopKTrainingSAEConfig(
        d_in=d_in, d_sae=6, k=2, matryoshka_widths=[3, 6], use_matryoshka_aux_loss=True,
        rescale_acts_by_decoder_norm=False))
    _rand(sae)
    x = torch.randn(2, d_in)
    pre = x @ sae.W_enc + sae.b_enc
    dead = torch.zeros(6, dtype=torch.bool)
    dead[1] = True
    dead[3:6] = True
    acts = sae.activation_fn(pre)
    out = acts @ sae.W_dec + sae.b_dec
    W = sae.W_dec.data
    total = 0.0
    partial = sae.b_dec.data
    for lo, hi in ((0, 3), (3, 6)):
        partial = partial + acts[:, lo:hi] @ W[lo:hi]
        nd = int(dead[lo:hi].sum())
        a = calculate_topk_aux_acts(min(k_aux, nd), pre[:, lo:hi], dead[lo:hi])
        total = total + min(nd / k_aux, 1.0) * ((a @ W[lo:hi] - (x - partial)) ** 2).sum(-1).mean()
    got = sae.calculate_matryoshka_aux_loss(x, out, acts, pre, dead)
    assert got.item() == pytest.approx((sae.cfg.aux_loss_coefficient * total).item(), rel=1e-5)


def test_matryoshka_aux_loss_flag_off_matches_base_class_and_levels_without_dead_skip():
    cfg = dict(d_in=8, d_sae=12, k=2, matryoshka_widths=[4, 12], rescale_acts_by_decoder_norm=False)
    off = MatryoshkaBatchTopKTrainingSAE(MatryoshkaBatchTopKTrainingSAEConfig(**cfg))
    on = MatryoshkaBatchTopKTrainingSAE(MatryoshkaBatchTopKTrainingSAEConfig(**cfg, use_matryoshka_aux_loss=True))
    _rand(off)
    on.load_state_dict(off.state_dict())
    x = torch.randn(10, 8)
    dead = torch.zeros(12, dtype=torch.bool)
    dead[6:] = True  # only the outer level has dead latents
    with torch.no_grad():
        f, pre = off.encode_with_hidden_pre(x)
        y = off.decode(f)
        a_off = off.calculate_aux_loss(_step(x, dead), f, pre, y)["auxiliary_reconstruction_loss"]
        torch.testing.assert_close(a_off, off.calculate_topk_aux_loss(x, y, pre, dead))
        a_on = on.calculate_matryoshka_aux_loss(x, y, f, pre, dead)
        # one level contributes: its residual is the full reconstruction's
        nd = 6
        a = calculate_topk_aux_acts(4, pre[:, 4:], dead[4:])
        want = on.cfg.aux_loss_coefficient * min(nd / 4, 1.0) * ((a @ on.W_dec[4:] - (x - y)) ** 2).sum(-1).mean()
        torch.testing.assert_close(a_on, want, rtol=1e-5, atol=1e-6)
    assert on.calculate_matryoshka_aux_loss(x, y, f, pre, torch.zeros(12, dtype=torch.bool)).item() == 0.0


def test_matryoshka_aux_loss_gradients_reach_own_level_decoder_rows():
    sae = MatryoshkaBatchTopKTrainingSAE(MatryoshkaBatchTopKTrainingSAEConfig(
        d_in=8, d_sae=12, k=2, matryoshka_widths=[4, 12], use_matryoshka_aux_loss=True,
        rescale_acts_by_decoder_norm=False))
    _rand(sae)
    x = torch.randn(10, 8)
    dead = torch.zeros(12, dtype=torch.bool)
    dead[:2] = True  # dead latents only in the first level
    f, pre = sae.encode_with_hidden_pre(x)
    y = sae.decode(f).detach()
    sae.zero_grad()
    sae.calculate_matryoshka_aux_loss(x, y, f.detach(), pre, dead).backward()
    g = sae.W_dec.grad
    assert g[:2].abs().sum() > 0 and g[4:].abs().sum() == 0
