"""Gated and Standard SAEs (behaviour of sae_lens/saes/gated_sae.py and standard_sae.py; expected
values follow tests/saes/test_gated_sae.py and test_standard_sae.py)."""

import pytest
import torch

from saelens_b200.models.gated import GatedSAE, GatedSAEConfig, GatedTrainingSAE, GatedTrainingSAEConfig
from saelens_b200.models.sae import SAE, TrainStepInput
from saelens_b200.models.standard import (
    StandardSAE,
    StandardSAEConfig,
    StandardTrainingSAE,
    StandardTrainingSAEConfig,
)


def _step(x, **coef):
    return TrainStepInput(sae_in=x, coefficients=coef, dead_neuron_mask=None, n_training_steps=0,
                          is_logging_step=False)


@pytest.mark.parametrize("use_error_term", [True, False])
def test_gated_forward_values(use_error_term):
    sae = GatedSAE(GatedSAEConfig(d_in=2, d_sae=3))
    sae._use_error_term = use_error_term
    with torch.no_grad():
        sae.W_enc.fill_(1.0)
        sae.W_dec.fill_(1.0)
        sae.b_dec.zero_()
        sae.b_gate.copy_(torch.tensor([-2.0, 0.0, 1.0]))
        sae.r_mag.copy_(torch.tensor([1.0, 2.0, 3.0]))
        sae.b_mag.fill_(1.0)
    x = torch.tensor([[0.3, 0.3]])
    recons = torch.tensor([[18.4848, 18.4848]])
    out, cache = sae.run_with_cache(x)
    torch.testing.assert_close(out, x if use_error_term else recons, atol=1e-3, rtol=0)
    torch.testing.assert_close(cache["hook_sae_input"], x)
    torch.testing.assert_close(cache["hook_sae_recons"], recons, atol=1e-3, rtol=0)
    torch.testing.assert_close(cache["hook_sae_acts_pre"], torch.tensor([[2.6310, 5.4334, 13.0513]]), atol=1e-3,
                               rtol=0)
    torch.testing.assert_close(cache["hook_sae_acts_post"], torch.tensor([[0.0, 5.4334, 13.0513]]), atol=1e-3,
                               rtol=0)
    if use_error_term:
        torch.testing.assert_close(cache["hook_sae_error"], x - recons, atol=1e-3, rtol=0)


def test_gated_training_encoding_and_loss():
    torch.manual_seed(0)
    sae = GatedTrainingSAE(GatedTrainingSAEConfig(d_in=8, d_sae=16, l1_coefficient=0.7, decoder_init_norm=1.0))
    x = torch.randn(32, 8)
    f, pre = sae.encode_with_hidden_pre(x)
    xc = x - sae.b_dec
    gate = (xc @ sae.W_enc + sae.b_gate > 0).float()
    mag = torch.relu(xc @ (sae.W_enc * sae.r_mag.exp()) + sae.b_mag)
    torch.testing.assert_close(f, gate * mag, atol=1e-6, rtol=1e-5)
    out = sae.training_forward_pass(_step(x, l1=0.7))
    via_gate = torch.relu(xc @ sae.W_enc + sae.b_gate)
    l1 = 0.7 * (via_gate * sae.W_dec.norm(dim=-1)).sum(-1).mean()
    aux = ((via_gate @ sae.W_dec + sae.b_dec - x) ** 2).sum(-1).mean()
    assert out.loss.item() == pytest.approx((out.losses["mse_loss"] + l1 + aux).item(), rel=1e-4)


def test_gated_save_load_and_export(tmp_path):
    torch.manual_seed(0)
    sae = GatedSAE(GatedSAEConfig(d_in=8, d_sae=16))
    with torch.no_grad():
        for p in sae.parameters():
            p.copy_(torch.randn_like(p) * 0.3)
    sae.save_model(tmp_path / "inf")
    back = SAE.load_from_pretrained(tmp_path / "inf")
    assert isinstance(back, GatedSAE)
    x = torch.randn(10, 8)
    with torch.no_grad():
        torch.testing.assert_close(back(x), sae(x))
    tr = GatedTrainingSAE(GatedTrainingSAEConfig(d_in=8, d_sae=16))
    tr.save_inference_model(tmp_path / "tr")
    inf = SAE.load_from_disk(tmp_path / "tr")
    assert isinstance(inf, GatedSAE)
    with torch.no_grad():
        torch.testing.assert_close(inf(x), tr.decode(tr.encode(x)), rtol=1e-4, atol=1e-5)


def test_standard_forward_and_l1_loss():
    torch.manual_seed(0)
    sae = StandardTrainingSAE(StandardTrainingSAEConfig(d_in=8, d_sae=16, l1_coefficient=2.0, lp_norm=1.0))
    x = torch.randn(12, 8)
    out = sae.training_forward_pass(_step(x, l1=2.0))
    f = torch.relu((x - sae.b_dec) @ sae.W_enc + sae.b_enc)
    torch.testing.assert_close(out.feature_acts, f)
    torch.testing.assert_close(out.losses["l1_loss"], 2.0 * (f * sae.W_dec.norm(dim=-1)).norm(p=1, dim=-1).mean())
    torch.testing.assert_close(out.losses["mse_loss"], ((f @ sae.W_dec + sae.b_dec - x) ** 2).sum(-1).mean())


def test_standard_initialization_options():
    sae = StandardTrainingSAE(StandardTrainingSAEConfig(d_in=8, d_sae=16, decoder_init_norm=0.1))
    torch.testing.assert_close(sae.W_dec.norm(dim=-1), torch.full((16,), 0.1), rtol=1e-5, atol=1e-6)
    torch.testing.assert_close(sae.W_enc, sae.W_dec.T)
    assert torch.all(sae.b_enc == 0) and torch.all(sae.b_dec == 0)
    sae = StandardTrainingSAE(StandardTrainingSAEConfig(d_in=8, d_sae=16, decoder_init_norm=None))
    torch.testing.assert_close(sae.W_enc, sae.W_dec.T)


def test_standard_export_and_fold(tmp_path):
    torch.manual_seed(0)
    sae = StandardTrainingSAE(StandardTrainingSAEConfig(d_in=8, d_sae=16))
    with torch.no_grad():
        for p in sae.parameters():
            p.copy_(torch.randn_like(p) * 0.3)
    x = torch.randn(10, 8)
    sae.save_inference_model(tmp_path)
    inf = SAE.load_from_disk(tmp_path)
    assert isinstance(inf, StandardSAE)
    with torch.no_grad():
        torch.testing.assert_close(inf(x), sae.decode(sae.encode(x)), rtol=1e-4, atol=1e-5)


def test_standard_inference_defaults():
    cfg = StandardSAEConfig(d_in=8, d_sae=16)
    sae = StandardSAE(cfg)
    assert sae.cfg.apply_b_dec_to_input and sae.cfg.normalize_activations == "none"
    assert sae.W_enc.shape == (8, 16) and sae.b_enc.shape == (16,)
