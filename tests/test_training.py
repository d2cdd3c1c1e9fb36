"""CPU tests: trainer loop, schedules, mixing buffer, activation scaler, checkpoint/resume."""

import json
import math

import pytest
import torch

from saelens_b200.config import LoggingConfig, SAETrainerConfig
from saelens_b200.models.standard import StandardTrainingSAE, StandardTrainingSAEConfig
from saelens_b200.models.topk import TopKTrainingSAE, TopKTrainingSAEConfig
from saelens_b200.training.activation_scaler import ActivationScaler
from saelens_b200.training.mixing_buffer import mixing_buffer
from saelens_b200.training.optim import CoefficientScheduler, LRSchedule, get_lr_scheduler
from saelens_b200.training.sae_trainer import SAETrainer


def _trainer_cfg(tmp_path=None, steps=20, batch=32, **kw):
    base = dict(
        n_checkpoints=0, checkpoint_path=str(tmp_path / "ckpt") if tmp_path else None,
        save_final_checkpoint=False, output_path=str(tmp_path / "out") if tmp_path else None,
        save_mse_every_n_steps=0, save_timing_every_n_steps=0, save_memory_every_n_steps=0,
        synchronize_timing=False, multi_sae_backward_order="forward", multi_sae_stats_sync_mode="immediate",
        multi_sae_stats_sync_interval=1, total_training_samples=steps * batch, device="cpu", autocast=False,
        lr=1e-3, lr_end=1e-4, lr_scheduler_name="constant", lr_warm_up_steps=0, adam_beta1=0.9, adam_beta2=0.999,
        lr_decay_steps=0, n_restart_cycles=1, train_batch_size_samples=batch, dead_feature_window=5,
        feature_sampling_window=10, logger=LoggingConfig(log_to_wandb=False),
    )
    base.update(kw)
    return SAETrainerConfig(**base)


def _data(d_in=16, batch=32, seed=0):
    g = torch.Generator().manual_seed(seed)
    basis = torch.randn(8, d_in, generator=g)

    def gen():
        while True:
            c = torch.relu(torch.randn(batch, 8, generator=g))
            yield c @ basis

    return gen()


@pytest.mark.parametrize("name", ["constant", "cosineannealing", "cosineannealingwarmrestarts"])
@pytest.mark.parametrize("warm,decay", [(0, 0), (5, 0), (0, 6), (4, 5)])
def test_lr_schedule_matches_torch_chain(name, warm, decay):
    steps, lr, lr_end = 40, 1e-3, 1e-4
    p = torch.nn.Parameter(torch.zeros(1))
    opt = torch.optim.Adam([p], lr=lr)
    sched = get_lr_scheduler(name, opt, steps, lr, warm, decay, lr_end, 2)
    mine = LRSchedule(name, steps, lr, warm, decay, lr_end, 2)
    for t in range(steps):
        assert opt.param_groups[0]["lr"] == pytest.approx(mine.lr_at(t), rel=1e-6, abs=1e-12), t
        opt.step()
        sched.step()


def test_coefficient_scheduler_warmup():
    s = CoefficientScheduler(warm_up_steps=4, final_value=2.0)
    vals = [s.value] + [s.step() for _ in range(6)]
    assert vals[0] == 0.0 and vals[1] == pytest.approx(0.5) and vals[4] == pytest.approx(2.0)
    assert vals[-1] == 2.0


def test_mixing_buffer_serves_every_row_once():
    batches = [torch.arange(i * 10, (i + 1) * 10).float().unsqueeze(1) for i in range(10)]
    out = list(mixing_buffer(buffer_size=30, batch_size=5, activations_loader=iter(batches), mix_fraction=0.5,
                             generator=torch.Generator().manual_seed(0)))
    served = torch.cat(out).flatten().sort().values
    assert torch.equal(served, torch.arange(100).float())
    assert all(b.shape[0] == 5 for b in out)


def test_mixing_buffer_no_mix_is_in_order():
    batches = [torch.arange(i * 4, (i + 1) * 4).float().unsqueeze(1) for i in range(4)]
    out = torch.cat(list(mixing_buffer(8, 4, iter(batches), mix_fraction=0.0))).flatten()
    assert torch.equal(out, torch.arange(16).float())


def test_mixing_buffer_dict_batches_stay_aligned():
    batches = [{"a": torch.arange(i * 6, (i + 1) * 6).float(), "b": -torch.arange(i * 6, (i + 1) * 6).float()}
               for i in range(4)]
    for b in mixing_buffer(12, 4, iter(batches), mix_fraction=0.5):
        assert torch.equal(b["a"], -b["b"])


def test_activation_scaler(tmp_path):
    s = ActivationScaler()
    data = iter([torch.ones(4, 16) * 2.0] * 10)
    s.estimate_scaling_factor(16, data, n_batches_for_norm_estimate=5)
    assert s.scaling_factor == pytest.approx(math.sqrt(16) / 8.0)
    s.save(str(tmp_path / "a.json"))
    t = ActivationScaler()
    t.load(tmp_path / "a.json")
    assert t.scaling_factor == s.scaling_factor
    with pytest.raises(ValueError):
        s.save(str(tmp_path / "a.txt"))


def test_trainer_reduces_loss_standard(tmp_path):
    sae = StandardTrainingSAE(StandardTrainingSAEConfig(d_in=16, d_sae=64, l1_coefficient=1e-3))
    cfg = _trainer_cfg(tmp_path, steps=60, save_mse_every_n_steps=1)
    tr = SAETrainer(cfg, sae, _data())
    assert tr.engine is None
    tr.fit()
    rows = [json.loads(x) for x in (tmp_path / "out" / "mse_history.jsonl").read_text().splitlines()]
    assert len(rows) == 60
    assert rows[-1]["mse_loss"] < 0.5 * rows[0]["mse_loss"]


def test_trainer_topk_dead_tracking_and_aux(tmp_path):
    sae = TopKTrainingSAE(TopKTrainingSAEConfig(d_in=16, d_sae=64, k=2))
    tr = SAETrainer(_trainer_cfg(tmp_path, steps=12), sae, _data())
    tr.fit()
    assert tr.n_training_steps == 12
    assert tr.n_forward_passes_since_fired.max() <= 12
    assert tr.dead_neurons.dtype == torch.bool


def test_checkpoint_and_resume_roundtrip(tmp_path):
    sae = StandardTrainingSAE(StandardTrainingSAEConfig(d_in=16, d_sae=32))
    tr = SAETrainer(_trainer_cfg(tmp_path, steps=6), sae, _data())
    tr.fit_steps(6)
    tr.save_checkpoint("c1")
    ck = tmp_path / "ckpt" / "c1"
    for f in ("cfg.json", "sae_weights.safetensors", "sparsity.safetensors", "trainer_state.pt",
              "activation_scaler.json"):
        assert (ck / f).exists(), f
    sae2 = StandardTrainingSAE(StandardTrainingSAEConfig(d_in=16, d_sae=32))
    sae2.load_weights_from_checkpoint(ck)
    tr2 = SAETrainer(_trainer_cfg(tmp_path, steps=6), sae2, _data())
    tr2.load_trainer_state(ck)
    assert tr2.n_training_steps == 6
    st1 = tr.optimizer.state[tr.sae.W_enc]["exp_avg"]
    st2 = tr2.optimizer.state[tr2.sae.W_enc]["exp_avg"]
    assert torch.allclose(st1, st2)
    for k, v in sae.state_dict().items():
        assert torch.allclose(sae2.state_dict()[k], v)


def test_resume_rejects_mode_mismatch(tmp_path):
    sae = StandardTrainingSAE(StandardTrainingSAEConfig(d_in=16, d_sae=32))
    tr = SAETrainer(_trainer_cfg(tmp_path, steps=2), sae, _data())
    tr.fit_steps(2)
    tr.save_checkpoint("c")
    state = torch.load(tmp_path / "ckpt" / "c" / "trainer_state.pt", weights_only=False)
    state["sae_dp_mode"] = "ddp"
    torch.save(state, tmp_path / "ckpt" / "c" / "trainer_state.pt")
    with pytest.raises(ValueError, match="Cross-mode"):
        tr.load_trainer_state(tmp_path / "ckpt" / "c")


def test_n_checkpoints_thresholds(tmp_path):
    sae = StandardTrainingSAE(StandardTrainingSAEConfig(d_in=16, d_sae=32))
    tr = SAETrainer(_trainer_cfg(tmp_path, steps=10, n_checkpoints=2), sae, _data())
    tr.fit()
    ckpts = sorted(p.name for p in (tmp_path / "ckpt").iterdir())
    assert len(ckpts) == 2


def test_quiesce_file_stops_and_checkpoints(tmp_path):
    sae = StandardTrainingSAE(StandardTrainingSAEConfig(d_in=16, d_sae=32))
    req = tmp_path / "quiesce_request"
    ack = tmp_path / "quiesce_ack"
    req.touch()
    tr = SAETrainer(_trainer_cfg(tmp_path, steps=10), sae, _data())
    tr.fit(quiesce_request_path=req, quiesce_ack_path=ack)
    assert tr.n_training_steps == 1
    assert ack.exists()
    assert any(p.name.startswith("quiesce_") for p in (tmp_path / "ckpt").iterdir())


def test_timing_and_memory_histories(tmp_path):
    sae = StandardTrainingSAE(StandardTrainingSAEConfig(d_in=16, d_sae=32))
    tr = SAETrainer(_trainer_cfg(tmp_path, steps=4, save_timing_every_n_steps=2), sae, _data())
    tr.fit()
    rows = (tmp_path / "out" / "timing_history.jsonl").read_text().splitlines()
    assert len(rows) == 2 and "sae_time_s" in json.loads(rows[0])


def test_wandb_shim_offline_logging(tmp_path, monkeypatch):
    monkeypatch.setenv("SAELENS_B200_WANDB_DIR", str(tmp_path / "wb"))
    sae = StandardTrainingSAE(StandardTrainingSAEConfig(d_in=16, d_sae=32))
    cfg = _trainer_cfg(tmp_path, steps=20, logger=LoggingConfig(log_to_wandb=True, wandb_log_frequency=5,
                                                                eval_every_n_wandb_logs=2))
    tr = SAETrainer(cfg, sae, _data())
    tr.fit()
    from saelens_b200.utils import wandb_shim

    if not wandb_shim._live():
        lines = (tmp_path / "wb" / "wandb_log.jsonl").read_text().splitlines()
        assert any('"metrics/l0"' in ln for ln in lines)
