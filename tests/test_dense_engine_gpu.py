"""Native Standard (ReLU + L1 weighted by decoder norms) and Gated training steps against fp32
autograd of the PyTorch training SAEs (MSE + L1 [+ the gated auxiliary reconstruction]), on the
same bf16 weights: losses, every parameter gradient, and a few optimisation steps."""

import pytest
import torch

pytestmark = pytest.mark.gpu


def _rel(a, b):
    return ((a.float() - b.float()).norm() / (b.float().norm() + 1e-12)).item()


def _perturb(sae):
    with torch.no_grad():
        for name, p in sae.named_parameters():
            if p.dim() == 1:
                p.normal_(0, 0.05)
        sae.W_enc.mul_(3.0)


@pytest.mark.parametrize("arch", ["standard", "gated"])
def test_dense_engine_matches_autograd(arch):
    from saelens_b200.models.gated import GatedTrainingSAE, GatedTrainingSAEConfig
    from saelens_b200.models.sae import TrainStepInput
    from saelens_b200.models.standard import StandardTrainingSAE, StandardTrainingSAEConfig
    from saelens_b200.training.dense_engine import GatedEngine, StandardEngine, dense_engine_class

    torch.manual_seed(0)
    cls, cfg_cls, eng_cls = ((StandardTrainingSAE, StandardTrainingSAEConfig, StandardEngine) if arch == "standard"
                             else (GatedTrainingSAE, GatedTrainingSAEConfig, GatedEngine))
    kw = dict(d_in=256, d_sae=2048, l1_coefficient=0.5, device="cuda")
    sae = cls(cfg_cls(**kw))
    _perturb(sae)
    assert dense_engine_class(sae) is eng_cls
    x = torch.randn(512, 256, device="cuda").to(torch.bfloat16)
    eng = eng_cls(sae, lr=1e-3)
    # fp32 oracle on the bf16 compute copies and the fp32 vectors
    ref = cls(cfg_cls(dtype="float32", **kw))
    with torch.no_grad():
        ref.W_enc.copy_(eng.w_enc.float().T)
        ref.W_dec.copy_(eng.w_dec.float())
        ref.b_dec.copy_(eng.p_bdec)
        if arch == "standard":
            ref.b_enc.copy_(eng.p_benc)
        else:
            ref.b_mag.copy_(eng.p_benc)
            ref.b_gate.copy_(eng.p_bgate)
            ref.r_mag.copy_(eng.p_rmag)
    res = eng.step(x, update=False)
    torch.cuda.synchronize()
    eng.status.check()
    out = ref.training_forward_pass(TrainStepInput(sae_in=x.float(), coefficients={"l1": 0.5}, dead_neuron_mask=None,
                                                   n_training_steps=0))
    out.loss.backward()
    assert abs(res.mse_loss.item() - out.losses["mse_loss"].item()) <= 2e-2 * out.losses["mse_loss"].item()
    assert abs(res.aux_loss.item() - out.losses["l1_loss"].item()) <= 2e-2 * out.losses["l1_loss"].item()
    if arch == "gated":
        want = out.losses["auxiliary_reconstruction_loss"].item()
        assert abs(res.extra_losses["auxiliary_reconstruction_loss"].item() - want) <= 2e-2 * want
    assert _rel(eng.g_dec, ref.W_dec.grad) < 3e-2
    assert _rel(eng.g_enc, ref.W_enc.grad.T) < 3e-2
    if arch == "standard":
        assert _rel(eng.g_benc, ref.b_enc.grad) < 3e-2
    else:
        assert _rel(eng.g_benc, ref.b_mag.grad) < 3e-2
        assert _rel(eng.g_bgate, ref.b_gate.grad) < 3e-2
        assert _rel(eng.g_rmag, ref.r_mag.grad) < 5e-2
    losses = [float(eng.step(x).loss) for _ in range(5)]
    assert losses[-1] < losses[0]


def test_trainer_picks_the_dense_engines():
    from saelens_b200.config import LoggingConfig, SAETrainerConfig
    from saelens_b200.models.gated import GatedTrainingSAE, GatedTrainingSAEConfig
    from saelens_b200.models.standard import StandardTrainingSAE, StandardTrainingSAEConfig
    from saelens_b200.training.dense_engine import GatedEngine, StandardEngine
    from saelens_b200.training.sae_trainer import SAETrainer

    cfg = SAETrainerConfig(
        n_checkpoints=0, checkpoint_path=None, save_final_checkpoint=False, output_path=None,
        save_mse_every_n_steps=0, save_timing_every_n_steps=0, save_memory_every_n_steps=0, synchronize_timing=False,
        multi_sae_backward_order="forward", multi_sae_stats_sync_mode="immediate", multi_sae_stats_sync_interval=1,
        total_training_samples=256 * 3, device="cuda", autocast=False, lr=1e-3, lr_end=1e-4,
        lr_scheduler_name="constant", lr_warm_up_steps=0, adam_beta1=0.9, adam_beta2=0.999, lr_decay_steps=0,
        n_restart_cycles=1, train_batch_size_samples=256, dead_feature_window=1000, feature_sampling_window=2000,
        logger=LoggingConfig(log_to_wandb=False))
    for cls, cfg_cls, eng_cls in ((StandardTrainingSAE, StandardTrainingSAEConfig, StandardEngine),
                                  (GatedTrainingSAE, GatedTrainingSAEConfig, GatedEngine)):
        sae = cls(cfg_cls(d_in=256, d_sae=1024, device="cuda"))
        tr = SAETrainer(cfg, sae, iter([torch.randn(256, 256, device="cuda") for _ in range(3)]))
        assert isinstance(tr.engine, eng_cls)
        losses = tr.fit_steps(3)
        assert len(losses) == 3 and all(v == v for v in losses)
