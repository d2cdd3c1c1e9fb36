"""MultiSAETrainer checkpoints under SAE tensor parallelism (2 gloo ranks, TopK SAEs sharded over
latents): periodic checkpoints, a saved checkpoint holds the full gathered weights, and resuming
into freshly initialised shards restores every rank's weight shard, per-latent statistics and Adam
moments (the weights are read by the first TP rank and scattered)."""

import json
import os
import socket

import torch
import torch.multiprocessing as mp


def _port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _cfg(tmp):
    from saelens_b200.config import LoggingConfig, SAETrainerConfig

    return SAETrainerConfig(
        n_checkpoints=1, checkpoint_path=os.path.join(tmp, "ckpts"), save_final_checkpoint=False, output_path=None,
        save_mse_every_n_steps=0, save_timing_every_n_steps=0, save_memory_every_n_steps=0, synchronize_timing=False,
        multi_sae_backward_order="forward", multi_sae_stats_sync_mode="immediate", multi_sae_stats_sync_interval=1,
        total_training_samples=32 * 6, device="cpu", autocast=False, lr=1e-2, lr_end=1e-3,
        lr_scheduler_name="constant", lr_warm_up_steps=0, adam_beta1=0.9, adam_beta2=0.999, lr_decay_steps=0,
        n_restart_cycles=1, train_batch_size_samples=32, dead_feature_window=5, feature_sampling_window=100,
        logger=LoggingConfig(log_to_wandb=False))


def _saes(seed):
    import torch.distributed as dist

    from saelens_b200.models.topk import TopKTrainingSAE, TopKTrainingSAEConfig

    out = {}
    for i, h in enumerate(("blocks.0.hook_resid_post", "blocks.1.hook_resid_post")):
        torch.manual_seed(seed + i)
        sae = TopKTrainingSAE(TopKTrainingSAEConfig(d_in=16, d_sae=64, k=4))
        sae.shard_weights(dist.group.WORLD)
        out[h] = sae
    return out


def _worker(rank, world, port, tmp):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    import torch.distributed as dist

    dist.init_process_group("gloo", rank=rank, world_size=world)
    from saelens_b200.training.multi_sae_trainer import MultiSAETrainer

    hooks = ["blocks.0.hook_resid_post", "blocks.1.hook_resid_post"]
    g = torch.Generator().manual_seed(0)  # the same batches on both TP ranks

    def gen():
        while True:
            yield {h: torch.randn(32, 16, generator=g) for h in hooks}

    saes = _saes(10)
    tr = MultiSAETrainer(hook_names=hooks, sae_by_hook=saes, data_provider=gen(), cfg=_cfg(tmp))
    tr.fit()
    ck = tr.save_checkpoint(os.path.join(tmp, "manual"))
    want = {h: (saes[h].W_dec.detach().clone(), tr.act_freq_scores[h].clone(),
                tr.optimizer.state[saes[h].W_dec]["exp_avg"].clone()) for h in hooks}
    fresh = _saes(99)
    tr2 = MultiSAETrainer(hook_names=hooks, sae_by_hook=fresh, data_provider=gen(), cfg=_cfg(tmp))
    tr2.load_trainer_state(ck)
    ok = {}
    for h in hooks:
        w, f, m = want[h]
        ok[h] = [bool(torch.equal(fresh[h].W_dec, w)), bool(torch.equal(tr2.act_freq_scores[h], f)),
                 bool(torch.equal(tr2.optimizer.state[fresh[h].W_dec]["exp_avg"], m)),
                 int(fresh[h].W_dec.shape[0])]
    info = {"ok": ok, "steps": tr2.n_training_steps, "periodic": sorted(os.listdir(os.path.join(tmp, "ckpts")))}
    with open(os.path.join(tmp, f"r{rank}.json"), "w") as fh:
        json.dump(info, fh)
    dist.destroy_process_group()


def test_multi_sae_tp_checkpoint_round_trip(tmp_path):
    mp.spawn(_worker, args=(2, _port(), str(tmp_path)), nprocs=2, join=True)
    from safetensors.torch import load_file

    for r in range(2):
        info = json.loads((tmp_path / f"r{r}.json").read_text())
        assert info["steps"] == 6 and len(info["periodic"]) == 1
        for h, (w_ok, f_ok, m_ok, n_local) in info["ok"].items():
            assert w_ok and f_ok and m_ok and n_local == 32, (r, h)
    sd = load_file(str(tmp_path / "manual" / "blocks.0.hook_resid_post" / "sae_weights.safetensors"))
    assert sd["W_dec"].shape == (64, 16) and sd["W_enc"].shape == (16, 64)
