"""JumpReLU SAE (behaviour of sae_lens/saes/jumprelu_sae.py; expected values follow
tests/saes/test_jumprelu_sae.py): encoding, straight-through gradients, loss modes, pre-act loss,
folding and the inference export."""

import pytest
import torch

from saelens_b200.models.jumprelu import (
    JumpReLU,
    JumpReLUSAE,
    JumpReLUSAEConfig,
    JumpReLUTrainingSAE,
    JumpReLUTrainingSAEConfig,
    Step,
    calculate_pre_act_loss,
)
from saelens_b200.models.sae import SAE, TrainStepInput


def _step(x, l0=1.0, dead=None):
    return TrainStepInput(sae_in=x, coefficients={"l0": l0}, dead_neuron_mask=dead, n_training_steps=0,
                          is_logging_step=False)


def _sae(**kw):
    torch.manual_seed(0)
    cfg = JumpReLUTrainingSAEConfig(d_in=8, d_sae=16, **kw)
    sae = JumpReLUTrainingSAE(cfg)
    with torch.no_grad():
        sae.W_enc.normal_(0, 0.5)
        sae.b_enc.normal_(0, 0.1)
    return sae


def test_training_encoding_is_thresholded_relu():
    sae = _sae(jumprelu_init_threshold=0.1)
    x = torch.randn(5, 8)
    f, pre = sae.encode_with_hidden_pre(x)
    want_pre = (x - sae.b_dec) @ sae.W_enc + sae.b_enc
    torch.testing.assert_close(pre, want_pre)
    torch.testing.assert_close(f, torch.where(pre > sae.threshold, pre, torch.zeros_like(pre)))


def test_step_and_jumprelu_straight_through_gradients():
    # inputs are [batch, d_sae]; threshold gradients are summed over the batch
    x = torch.tensor([[0.2, 0.5, 0.9], [0.2, 0.45, 0.9]], requires_grad=True)
    th = torch.tensor([0.5, 0.5, 0.5], requires_grad=True)
    bw = 0.2
    y = JumpReLU.apply(x, th, bw)
    torch.testing.assert_close(y.detach(), torch.tensor([[0.0, 0.0, 0.9], [0.0, 0.0, 0.9]]))
    y.sum().backward()
    # dy/dx = 1 above threshold; dy/dth = -(th / bw) * rect((x - th) / bw)
    torch.testing.assert_close(x.grad, torch.tensor([[0.0, 0.0, 1.0], [0.0, 0.0, 1.0]]))
    torch.testing.assert_close(th.grad, torch.tensor([0.0, -2 * 0.5 / 0.2, 0.0]))
    x2 = torch.tensor([[0.2, 0.55, 0.9]], requires_grad=True)
    th2 = torch.tensor([0.5, 0.5, 0.5], requires_grad=True)
    s = Step.apply(x2, th2, bw)
    torch.testing.assert_close(s.detach(), torch.tensor([[0.0, 1.0, 1.0]]))
    s.sum().backward()
    torch.testing.assert_close(th2.grad, torch.tensor([0.0, -1 / 0.2, 0.0]))


def test_training_forward_pass_step_mode_losses():
    sae = _sae(l0_coefficient=0.3)
    x = torch.randn(6, 8)
    out = sae.training_forward_pass(_step(x, l0=0.3))
    f = out.feature_acts
    mse = ((out.sae_out - x) ** 2).sum(-1).mean()
    torch.testing.assert_close(out.losses["mse_loss"], mse)
    l0 = (f > 0).float().sum(-1).mean() * 0.3
    torch.testing.assert_close(out.losses["l0_loss"], l0)
    torch.testing.assert_close(out.loss, mse + l0)


def test_pre_act_loss_zero_without_dead_mask():
    assert float(calculate_pre_act_loss(0.5, torch.ones(8) * 0.5, torch.randn(4, 8), None, torch.ones(8))) == 0.0


def test_pre_act_loss_values():
    loss = calculate_pre_act_loss(1.0, torch.tensor([1.0, 2.0, 1.5, 0.5]),
                                  torch.tensor([[0.5, 1.5, 1.0, 0.8], [0.8, 2.5, 1.2, 0.2]]),
                                  torch.tensor([1.0, 0.0, 1.0, 0.0]), torch.tensor([2.0, 1.0, 1.5, 3.0]))
    torch.testing.assert_close(loss, torch.tensor(1.3))


def test_tanh_mode_with_pre_act_loss_sums_components():
    sae = _sae(jumprelu_sparsity_loss_mode="tanh", pre_act_loss_coefficient=0.1, l0_coefficient=0.5)
    dead = torch.zeros(16)
    dead[0] = dead[2] = 1.0
    out = sae.training_forward_pass(_step(torch.randn(4, 8), l0=0.5, dead=dead))
    assert out.sae_out.shape == (4, 8) and out.feature_acts.shape == (4, 16)
    torch.testing.assert_close(out.loss, out.losses["mse_loss"] + out.losses["l0_loss"] + out.losses["pre_act_loss"])
    assert out.losses["pre_act_loss"] >= 0


def test_tanh_scale_increases_l0_loss():
    small = _sae(jumprelu_sparsity_loss_mode="tanh", jumprelu_tanh_scale=2.0)
    large = _sae(jumprelu_sparsity_loss_mode="tanh", jumprelu_tanh_scale=8.0)
    large.load_state_dict(small.state_dict())
    x = torch.randn(4, 8)
    a, b = small.training_forward_pass(_step(x)), large.training_forward_pass(_step(x))
    assert b.losses["l0_loss"] > a.losses["l0_loss"]
    torch.testing.assert_close(a.feature_acts, b.feature_acts)


def test_invalid_sparsity_mode_raises():
    sae = _sae(jumprelu_sparsity_loss_mode="nonsense")
    with pytest.raises(ValueError):
        sae.training_forward_pass(_step(torch.randn(8, 8)))


def test_initialization_threshold_and_shapes():
    sae = JumpReLUTrainingSAE(JumpReLUTrainingSAEConfig(d_in=8, d_sae=16, jumprelu_init_threshold=0.01))
    torch.testing.assert_close(sae.threshold, torch.full((16,), 0.01))
    assert sae.log_threshold.shape == (16,) and sae.W_enc.shape == (8, 16) and sae.W_dec.shape == (16, 8)
    inf = JumpReLUSAE(JumpReLUSAEConfig(d_in=8, d_sae=16))
    assert inf.threshold.shape == (16,)


@pytest.mark.parametrize("use_error_term", [True, False])
def test_inference_forward(use_error_term):
    torch.manual_seed(0)
    sae = JumpReLUSAE(JumpReLUSAEConfig(d_in=8, d_sae=16))
    with torch.no_grad():
        for p in sae.parameters():
            p.copy_(torch.rand_like(p) * 0.5)
    sae._use_error_term = use_error_term
    x = torch.randn(4, 8)
    with torch.no_grad():
        y = sae(x)
        pre = (x - sae.b_dec) @ sae.W_enc + sae.b_enc
        f = torch.where(pre > sae.threshold, pre, torch.zeros_like(pre))
        want = x if use_error_term else f @ sae.W_dec + sae.b_dec
    torch.testing.assert_close(y, want, rtol=1e-4, atol=1e-5)


def test_training_export_matches_inference_and_fold(tmp_path):
    sae = _sae(jumprelu_init_threshold=0.2)
    with torch.no_grad():
        sae.W_dec.mul_(3.0)
    x = torch.randn(10, 8)
    with torch.no_grad():
        y = sae.decode(sae.encode(x))
        sae.save_inference_model(tmp_path)
        inf = SAE.load_from_disk(tmp_path)
        assert isinstance(inf, JumpReLUSAE)
        torch.testing.assert_close(inf(x), y, rtol=1e-4, atol=1e-5)
        sae.fold_W_dec_norm()
        torch.testing.assert_close(sae.W_dec.norm(dim=-1), torch.ones(16))
        torch.testing.assert_close(sae.decode(sae.encode(x)), y, rtol=1e-4, atol=1e-5)
