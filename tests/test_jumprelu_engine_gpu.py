"""Native JumpReLU step against fp32 autograd of the JumpReLU training loss (MSE + step L0 with the
rectangle straight-through estimator for the threshold)."""

import pytest
import torch

pytestmark = pytest.mark.gpu


def _rel(a, b):
    return ((a.float() - b.float()).norm() / (b.float().norm() + 1e-12)).item()


def test_jumprelu_engine_matches_autograd():
    from saelens_b200.models.jumprelu import JumpReLUTrainingSAE, JumpReLUTrainingSAEConfig
    from saelens_b200.models.sae import TrainStepInput
    from saelens_b200.training.jumprelu_engine import JumpReLUEngine, jumprelu_engine_supported

    torch.manual_seed(0)
    cfg = JumpReLUTrainingSAEConfig(d_in=256, d_sae=2048, jumprelu_init_threshold=0.25, jumprelu_bandwidth=0.05,
                                    l0_coefficient=0.3, device="cuda")
    sae = JumpReLUTrainingSAE(cfg)
    with torch.no_grad():
        sae.b_enc.normal_(0, 0.01)
        sae.b_dec.normal_(0, 0.05)
        sae.W_enc.mul_(3.0)
        sae.log_threshold.add_(torch.randn_like(sae.log_threshold) * 0.2)
    assert jumprelu_engine_supported(sae)
    x = torch.randn(512, 256, device="cuda").to(torch.bfloat16)
    eng = JumpReLUEngine(sae, lr=1e-3)
    w_enc0, w_dec0 = eng.w_enc.float().clone(), eng.w_dec.float().clone()
    b_enc0, b_dec0, lthr0 = eng.p_benc.clone(), eng.p_bdec.clone(), eng.p_lthr.clone()
    res = eng.step(x, update=False)
    torch.cuda.synchronize()
    eng.status.check()
    assert int(eng.truncated.item()) == 0
    # fp32 oracle on the bf16 compute copies
    ref = JumpReLUTrainingSAE(JumpReLUTrainingSAEConfig(d_in=256, d_sae=2048, jumprelu_bandwidth=0.05,
                                                        l0_coefficient=0.3, device="cuda", dtype="float32"))
    with torch.no_grad():
        ref.W_enc.copy_(w_enc0.T)
        ref.W_dec.copy_(w_dec0)
        ref.b_enc.copy_(b_enc0)
        ref.b_dec.copy_(b_dec0)
        ref.log_threshold.copy_(lthr0)
    out = ref.training_forward_pass(TrainStepInput(sae_in=x.float(), coefficients={"l0": 0.3}, dead_neuron_mask=None,
                                                   n_training_steps=0))
    out.loss.backward()
    assert abs(res.mse_loss.item() - out.losses["mse_loss"].item()) <= 2e-2 * out.losses["mse_loss"].item()
    assert abs(res.aux_loss.item() - out.losses["l0_loss"].item()) <= 2e-2 * out.losses["l0_loss"].item()
    live = eng.colptr[1:] > eng.colptr[:-1]
    assert _rel(eng.g_dec[live], ref.W_dec.grad[live]) < 3e-2
    assert _rel(eng.g_enc[live], ref.W_enc.grad.T[live]) < 3e-2
    assert _rel(eng.g_benc, ref.b_enc.grad) < 3e-2
    assert _rel(eng.g_thr * lthr0.exp(), ref.log_threshold.grad) < 5e-2
    # a few optimisation steps lower the loss
    losses = [float(eng.step(x).loss) for _ in range(5)]
    assert losses[-1] < losses[0]
