"""Multi-process CPU (gloo) tests of the tensor- and data-parallel paths."""

import os
import socket
from datetime import timedelta

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _init(rank: int, world: int, port: int) -> None:
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))


def _topk_sae(k=4, d_in=8, d_sae=32):
    from saelens_b200.models.topk import TopKTrainingSAE, TopKTrainingSAEConfig

    torch.manual_seed(3)
    sae = TopKTrainingSAE(TopKTrainingSAEConfig(d_in=d_in, d_sae=d_sae, k=k))
    with torch.no_grad():
        sae.b_dec.normal_(0, 0.3)
        sae.b_enc.normal_(0, 0.1)
        sae.W_dec.mul_(torch.rand(d_sae, 1) + 0.5)
    return sae


def _tp_worker(rank, world, port, out_dir):
    from saelens_b200.models.sae import TrainStepInput

    _init(rank, world, port)
    sae = _topk_sae()
    sae.shard_weights(dist.group.WORLD)
    x = torch.randn(12, 8, generator=torch.Generator().manual_seed(5))
    dead = torch.zeros(32, dtype=torch.bool)
    dead[5:20] = True
    out = sae.training_forward_pass(TrainStepInput(sae_in=x, coefficients={}, dead_neuron_mask=dead))
    out.loss.backward()
    sae.sync_tensor_parallel_gradients()
    grads = {n: p.grad.clone() for n, p in sae.named_parameters()}
    total = sae.clip_grad_norm_(1e9)
    torch.save({"grads": grads, "loss": out.loss.item(), "norm": total.item()}, os.path.join(out_dir, f"tp{rank}.pt"))
    sae.save_model(os.path.join(out_dir, "tp_model"))
    dist.barrier()
    dist.destroy_process_group()


def test_topk_tp2_gradients_match_tp1(tmp_path):
    from saelens_b200.models.sae import TrainStepInput

    mp.spawn(_tp_worker, args=(2, _port(), str(tmp_path)), nprocs=2, join=True)
    sae = _topk_sae()
    x = torch.randn(12, 8, generator=torch.Generator().manual_seed(5))
    dead = torch.zeros(32, dtype=torch.bool)
    dead[5:20] = True
    out = sae.training_forward_pass(TrainStepInput(sae_in=x, coefficients={}, dead_neuron_mask=dead))
    out.loss.backward()
    full_norm = torch.sqrt(sum(p.grad.pow(2).sum() for p in sae.parameters()))
    dims = {"W_enc": 1, "W_dec": 0, "b_enc": 0, "b_dec": None}
    for r in range(2):
        res = torch.load(tmp_path / f"tp{r}.pt")
        assert res["loss"] == pytest.approx(out.loss.item(), rel=1e-5)
        assert res["norm"] == pytest.approx(full_norm.item(), rel=1e-4)
        for name, p in sae.named_parameters():
            d = dims[name]
            ref = p.grad if d is None else p.grad.narrow(d, r * 16, 16)
            assert torch.allclose(res["grads"][name], ref, atol=1e-5, rtol=1e-4), (r, name)
    # the TP save gathers the shards back into the full layout
    from saelens_b200.models.sae import TrainingSAE

    loaded = TrainingSAE.load_from_disk(tmp_path / "tp_model")
    assert torch.allclose(loaded.W_enc, sae.W_enc) and torch.allclose(loaded.W_dec, sae.W_dec)


def _dp_worker(rank, world, port, out_dir):
    from saelens_b200.config import LoggingConfig, SAETrainerConfig
    from saelens_b200.models.standard import StandardTrainingSAE, StandardTrainingSAEConfig
    from saelens_b200.training.sae_trainer import SAETrainer

    _init(rank, world, port)
    torch.manual_seed(0)
    sae = StandardTrainingSAE(StandardTrainingSAEConfig(d_in=8, d_sae=16))
    x = torch.randn(16, 8, generator=torch.Generator().manual_seed(9))
    rows = x[rank * 8 : (rank + 1) * 8]
    cfg = SAETrainerConfig(
        n_checkpoints=0, checkpoint_path=None, save_final_checkpoint=False, output_path=None,
        save_mse_every_n_steps=0, save_timing_every_n_steps=0, save_memory_every_n_steps=0,
        synchronize_timing=False, multi_sae_backward_order="forward", multi_sae_stats_sync_mode="immediate",
        multi_sae_stats_sync_interval=1, total_training_samples=8, device="cpu", autocast=False, lr=1e-2,
        lr_end=1e-3, lr_scheduler_name="constant", lr_warm_up_steps=0, adam_beta1=0.9, adam_beta2=0.999,
        lr_decay_steps=0, n_restart_cycles=1, train_batch_size_samples=8, dead_feature_window=5,
        feature_sampling_window=10, logger=LoggingConfig(log_to_wandb=False),
    )
    tr = SAETrainer(cfg, sae, iter([rows]), dp_group=dist.group.WORLD)
    tr.fit_steps(1)
    torch.save({k: v.clone() for k, v in sae.state_dict().items()}, os.path.join(out_dir, f"dp{rank}.pt"))
    dist.barrier()
    dist.destroy_process_group()


def test_manual_dp2_matches_single_process(tmp_path):
    from saelens_b200.models.standard import StandardTrainingSAE, StandardTrainingSAEConfig

    mp.spawn(_dp_worker, args=(2, _port(), str(tmp_path)), nprocs=2, join=True)
    torch.manual_seed(0)
    sae = StandardTrainingSAE(StandardTrainingSAEConfig(d_in=8, d_sae=16))
    x = torch.randn(16, 8, generator=torch.Generator().manual_seed(9))
    opt = torch.optim.Adam(sae.parameters(), lr=1e-2)
    from saelens_b200.models.sae import TrainStepInput

    # mean over the two halves' losses == DP mean of per-rank gradients
    loss = sum(sae.training_forward_pass(TrainStepInput(sae_in=h, coefficients={"l1": 1.0}, dead_neuron_mask=None)).loss
               for h in (x[:8], x[8:])) / 2
    loss.backward()
    torch.nn.utils.clip_grad_norm_(sae.parameters(), 1.0)
    opt.step()
    r0, r1 = torch.load(tmp_path / "dp0.pt"), torch.load(tmp_path / "dp1.pt")
    for k, v in sae.state_dict().items():
        assert torch.allclose(r0[k], r1[k])
        assert torch.allclose(r0[k], v, atol=1e-6), k
