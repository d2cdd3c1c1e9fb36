"""Native JumpReLU step, in its sparse and its dense form, against fp32 autograd of the JumpReLU
training loss (MSE + step L0 with the rectangle straight-through estimator for the threshold),
including the dense init of the reference's JumpReLU configs (threshold 0.001, every latent above
threshold in about half the rows)."""

import pytest
import torch

pytestmark = pytest.mark.gpu


def _rel(a, b):
    return ((a.float() - b.float()).norm() / (b.float().norm() + 1e-12)).item()


@pytest.mark.parametrize("mode, init_thr, bandwidth", [("sparse", 0.25, 0.05), ("dense", 0.25, 0.05),
                                                      ("dense", 0.001, 0.001)])
def test_jumprelu_engine_matches_autograd(mode, init_thr, bandwidth):
    from saelens_b200.models.jumprelu import JumpReLUTrainingSAE, JumpReLUTrainingSAEConfig
    from saelens_b200.models.sae import TrainStepInput
    from saelens_b200.training.jumprelu_engine import JumpReLUEngine, jumprelu_engine_supported

    torch.manual_seed(0)
    kw = dict(d_in=256, d_sae=2048, jumprelu_bandwidth=bandwidth, l0_coefficient=0.3, device="cuda")
    sae = JumpReLUTrainingSAE(JumpReLUTrainingSAEConfig(jumprelu_init_threshold=init_thr, **kw))
    with torch.no_grad():
        sae.b_enc.normal_(0, 0.01)
        sae.b_dec.normal_(0, 0.05)
        sae.W_enc.mul_(3.0)
        sae.log_threshold.add_(torch.randn_like(sae.log_threshold) * 0.2)
    assert jumprelu_engine_supported(sae)
    x = torch.randn(512, 256, device="cuda").to(torch.bfloat16)
    eng = JumpReLUEngine(sae, lr=1e-3, mode=mode)
    w_enc0, w_dec0 = eng.w_enc.float().clone(), eng.w_dec.float().clone()
    b_enc0, b_dec0, lthr0 = eng.p_benc.clone(), eng.p_bdec.clone(), eng.p_lthr.clone()
    res = eng.step(x, update=False)
    torch.cuda.synchronize()
    eng.status.check()
    assert (eng.sparse_steps, eng.dense_steps, eng.fallbacks) == ((1, 0, 0) if mode == "sparse" else (0, 1, 0))
    # fp32 oracle on the bf16 compute copies
    ref = JumpReLUTrainingSAE(JumpReLUTrainingSAEConfig(dtype="float32", **kw))
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
    live = (eng.colptr[1:] > eng.colptr[:-1]) if mode == "sparse" else torch.ones(2048, dtype=torch.bool,
                                                                                  device="cuda")
    assert _rel(eng.g_dec[live], ref.W_dec.grad[live]) < 3e-2
    assert _rel(eng.g_enc[live], ref.W_enc.grad.T[live]) < 3e-2
    assert _rel(eng.g_benc, ref.b_enc.grad) < 3e-2
    assert _rel(eng.g_thr * lthr0.exp(), ref.log_threshold.grad) < 5e-2
    # a few optimisation steps lower the loss
    losses = [float(eng.step(x).loss) for _ in range(5)]
    assert losses[-1] < losses[0]


def test_sparse_form_falls_back_to_dense_when_a_row_overflows_the_cap():
    from saelens_b200.models.jumprelu import JumpReLUTrainingSAE, JumpReLUTrainingSAEConfig
    from saelens_b200.training.jumprelu_engine import JumpReLUEngine

    torch.manual_seed(1)
    sae = JumpReLUTrainingSAE(JumpReLUTrainingSAEConfig(d_in=256, d_sae=4096, jumprelu_init_threshold=0.001,
                                                        jumprelu_bandwidth=0.001, device="cuda"))
    eng = JumpReLUEngine(sae, lr=1e-3, mode="sparse", cap=256)
    x = torch.randn(256, 256, device="cuda").to(torch.bfloat16)
    with pytest.warns(RuntimeWarning, match="running the dense form"):
        eng.step(x)
    assert (eng.sparse_steps, eng.dense_steps, eng.fallbacks) == (0, 1, 1) and eng.mode == "dense"


def test_trainer_uses_the_native_jumprelu_engine_by_default():
    from saelens_b200.config import LoggingConfig, SAETrainerConfig
    from saelens_b200.models.jumprelu import JumpReLUTrainingSAE, JumpReLUTrainingSAEConfig
    from saelens_b200.training.jumprelu_engine import JumpReLUEngine
    from saelens_b200.training.sae_trainer import SAETrainer

    sae = JumpReLUTrainingSAE(JumpReLUTrainingSAEConfig(d_in=256, d_sae=1024, device="cuda"))
    cfg = SAETrainerConfig(
        n_checkpoints=0, checkpoint_path=None, save_final_checkpoint=False, output_path=None,
        save_mse_every_n_steps=0, save_timing_every_n_steps=0, save_memory_every_n_steps=0, synchronize_timing=False,
        multi_sae_backward_order="forward", multi_sae_stats_sync_mode="immediate", multi_sae_stats_sync_interval=1,
        total_training_samples=256 * 4, device="cuda", autocast=False, lr=1e-3, lr_end=1e-4,
        lr_scheduler_name="constant", lr_warm_up_steps=0, adam_beta1=0.9, adam_beta2=0.999, lr_decay_steps=0,
        n_restart_cycles=1, train_batch_size_samples=256, dead_feature_window=1000, feature_sampling_window=2000,
        logger=LoggingConfig(log_to_wandb=False))
    data = iter([torch.randn(256, 256, device="cuda") for _ in range(4)])
    tr = SAETrainer(cfg, sae, data)
    assert isinstance(tr.engine, JumpReLUEngine)
    losses = tr.fit_steps(4)
    assert len(losses) == 4 and all(l == l for l in losses)
