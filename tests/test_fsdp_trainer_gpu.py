"""SAETrainer with sharded data parallel on the native engine (2 ranks): engine selection, the
gathered final weights, per-rank optimizer shards in checkpoints and resume."""

import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, out_dir):
    import torch.distributed as dist
    from datetime import timedelta

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    from saelens_b200.config import LoggingConfig, SAETrainerConfig
    from saelens_b200.models.topk import TopKTrainingSAE, TopKTrainingSAEConfig
    from saelens_b200.parallel.fsdp_engine import FSDPTopKEngine
    from saelens_b200.training.sae_trainer import SAETrainer

    dev = f"cuda:{rank}"

    def cfg(steps, ckpt):
        return SAETrainerConfig(
            n_checkpoints=0, checkpoint_path=ckpt, save_final_checkpoint=True, output_path=None,
            save_mse_every_n_steps=0, save_timing_every_n_steps=0, save_memory_every_n_steps=0,
            synchronize_timing=False, multi_sae_backward_order="forward", multi_sae_stats_sync_mode="immediate",
            multi_sae_stats_sync_interval=1, total_training_samples=steps * 256, device=dev, autocast=False,
            lr=1e-3, lr_end=1e-4, lr_scheduler_name="constant", lr_warm_up_steps=0, adam_beta1=0.9,
            adam_beta2=0.999, lr_decay_steps=0, n_restart_cycles=1, train_batch_size_samples=256,
            dead_feature_window=3, feature_sampling_window=4, logger=LoggingConfig(log_to_wandb=False))

    def data(seed):
        g = torch.Generator().manual_seed(seed)
        while True:
            yield torch.randn(256, 128, generator=g)

    def build():
        torch.manual_seed(3)
        return TopKTrainingSAE(TopKTrainingSAEConfig(d_in=128, d_sae=1024, k=16, device=dev))

    ckpt = os.path.join(out_dir, "ckpt")
    sae = build()
    tr = SAETrainer(cfg(6, ckpt), sae, data(rank), dp_group=dist.group.WORLD, native_fsdp=True)
    assert isinstance(tr.engine, FSDPTopKEngine) and tr.sae_dp_mode == "fsdp"
    out = tr.fit()
    assert out.W_dec.shape == (1024, 128) and out.W_enc.shape == (128, 1024)
    dist.barrier()
    final = sorted(p for p in os.listdir(ckpt) if p.startswith("final_"))[-1]
    state = torch.load(os.path.join(ckpt, final, "trainer_state.pt"), weights_only=False)
    # resume into a fresh sharded trainer
    sae2 = build()
    tr2 = SAETrainer(cfg(6, None), sae2, data(rank), dp_group=dist.group.WORLD, native_fsdp=True)
    from safetensors.torch import load_file

    sd = load_file(os.path.join(ckpt, final, "sae_weights.safetensors"))
    tr2.engine.load_weights(sd["W_enc"], sd["W_dec"], sd["b_enc"], sd["b_dec"])
    tr2.load_trainer_state(os.path.join(ckpt, final))
    same_m = torch.equal(tr2.engine.m_dec.cpu(), tr.engine.m_dec.cpu())
    torch.save({"W_dec": out.W_dec.detach().cpu(), "fmt": state["optimizer_state_format"], "same_m": same_m,
                "steps": tr2.n_training_steps, "saved_W_dec": sd["W_dec"]}, os.path.join(out_dir, f"r{rank}.pt"))
    tr.engine.close()
    tr2.engine.close()
    dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_trainer_native_fsdp_fit_save_resume(tmp_path):
    import torch.multiprocessing as mp

    mp.spawn(_worker, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True)
    r = [torch.load(tmp_path / f"r{i}.pt") for i in range(2)]
    assert torch.equal(r[0]["W_dec"], r[1]["W_dec"])  # the replicas agree after the gather
    assert torch.equal(r[0]["saved_W_dec"], r[0]["W_dec"])
    for x in r:
        assert x["fmt"] == "native_fsdp_latent_sharded" and x["same_m"] and x["steps"] == 6
