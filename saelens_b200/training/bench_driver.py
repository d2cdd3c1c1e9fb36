"""Measurement harness behind `bench.py` (device-timed and end-to-end tokens/s).

Kept in the package so the benchmark exercises exactly the code a user runs: the device-timed
loop drives `FusedTopKEngine.step` (or its tensor-parallel counterpart), the end-to-end loop drives
`SAETrainer.fit_steps` fed by a pinned-host-memory data provider.
"""

from __future__ import annotations

import gc
import math
from dataclasses import dataclass
from typing import Any

import torch
import torch.distributed as dist


@dataclass
class BenchSetup:
    d_in: int
    d_sae: int
    k: int
    batch: int
    world: int
    rank: int
    lr: float = 5e-5
    tp_exchange: str = "p2p"  # "p2p": fused NVLink kernels; "nccl": NCCL collectives between kernels
    arch: str = "topk"  # "topk" or "batchtopk" (k = mean active latents per row)


def _build_sae(s: BenchSetup) -> Any:
    from saelens_b200.models.batchtopk import BatchTopKTrainingSAE, BatchTopKTrainingSAEConfig
    from saelens_b200.models.topk import TopKTrainingSAE, TopKTrainingSAEConfig

    torch.manual_seed(1234)
    if s.arch == "batchtopk":
        return BatchTopKTrainingSAE(BatchTopKTrainingSAEConfig(d_in=s.d_in, d_sae=s.d_sae, k=s.k, dtype="bfloat16",
                                                               device="meta"))
    cfg = TopKTrainingSAEConfig(d_in=s.d_in, d_sae=s.d_sae, k=s.k, dtype="bfloat16", device="meta")
    sae = TopKTrainingSAE(cfg)
    return sae


def _materialise_local(sae: Any, s: BenchSetup) -> Any:
    """Random-init the local latent shard directly on the GPU (kaiming-uniform rows rescaled to
    the 0.1 decoder norm, encoder tied to the decoder transpose, zero biases)."""
    from torch import nn

    dev = torch.device("cuda", torch.cuda.current_device())
    n_local = s.d_sae // s.world
    g = torch.Generator(device=dev)
    g.manual_seed(1234 + s.rank)
    bound = math.sqrt(6.0 / s.d_in)  # kaiming_uniform_ on [d_sae, d_in]: gain sqrt(2), fan_in d_in
    W_dec = torch.empty(n_local, s.d_in, dtype=torch.bfloat16, device=dev).uniform_(-bound, bound, generator=g)
    W_dec = W_dec / W_dec.float().norm(dim=-1, keepdim=True).to(torch.bfloat16) * 0.1
    sae.cfg.device = str(dev)
    sae.W_dec = nn.Parameter(W_dec.contiguous(), requires_grad=False)
    sae.W_enc = nn.Parameter(W_dec.T, requires_grad=False)
    sae.b_enc = nn.Parameter(torch.zeros(n_local, dtype=torch.bfloat16, device=dev), requires_grad=False)
    sae.b_dec = nn.Parameter(torch.zeros(s.d_in, dtype=torch.bfloat16, device=dev), requires_grad=False)
    if hasattr(sae, "topk_threshold"):
        sae.topk_threshold = torch.zeros((), dtype=torch.double, device=dev)
    sae.device = dev
    return sae


def synthetic_batch(s: BenchSetup, seed: int, device: Any = "cpu", dtype: torch.dtype = torch.bfloat16) -> torch.Tensor:
    """N(0,1) activations rescaled to norm sqrt(d_in) (bf16 unless `dtype` says otherwise)."""
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    x = torch.randn(s.batch, s.d_in, generator=g, device=device)
    x = x / x.norm(dim=-1, keepdim=True) * math.sqrt(s.d_in)
    return x.to(dtype)


def _make_engine(s: BenchSetup) -> Any:
    sae = _materialise_local(_build_sae(s), s)
    if s.world == 1:
        from saelens_b200.training.engine import FusedTopKEngine

        return FusedTopKEngine(sae, lr=s.lr)
    from saelens_b200.parallel.tp_engine import TPTopKEngine

    return TPTopKEngine(sae, lr=s.lr, group=dist.group.WORLD, fused=s.tp_exchange == "p2p")


def _free(*objs: Any) -> None:
    for o in objs:
        del o
    gc.collect()
    torch.cuda.empty_cache()


def _max_over_ranks(v: float, world: int) -> float:
    if world == 1:
        return v
    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def _barrier(world: int) -> None:
    if world > 1:
        dist.barrier()


def run_device_timed(s: BenchSetup, steps: int, warmup: int, sampler: Any = None) -> dict[str, Any]:
    eng = _make_engine(s)
    dev = torch.device("cuda", torch.cuda.current_device())
    rows_local = s.batch // s.world if s.world > 1 else s.batch
    xs = [synthetic_batch(BenchSetup(**{**s.__dict__, "batch": rows_local}), seed=100 + 7 * i + s.rank, device=dev)
          for i in range(3)]
    for i in range(warmup):
        eng.step(xs[i % len(xs)])
    torch.cuda.synchronize()
    eng.status.check("warmup")
    launches0 = eng.launches
    _barrier(s.world)
    torch.cuda.synchronize()
    if sampler is not None:
        sampler.start()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record()
    for i in range(steps):
        eng.step(xs[i % len(xs)])
    t1.record()
    torch.cuda.synchronize()
    _barrier(s.world)
    clocks = sampler.stop() if sampler is not None else None
    eng.status.check("timed")
    ms = t0.elapsed_time(t1) / steps
    ms = _max_over_ranks(ms, s.world)
    launches = (eng.launches - launches0) // max(steps, 1)
    out = {"ms_per_step": ms, "gpu_launches": int(launches * steps), "clocks": clocks,
           "loss": float(eng.last_loss) if getattr(eng, "last_loss", None) is not None else None}
    if hasattr(eng, "close"):
        eng.close()
    del eng, xs
    _free()
    return out


class PinnedBatches:
    """Data provider serving pre-generated fp32 activation batches from pinned host memory, the
    dtype an activation store yields; the engine casts to bf16 on the device.  `n` distinct
    batches are served in turn."""

    N_DISTINCT = 8

    def __init__(self, s: BenchSetup, n: int = N_DISTINCT):
        self.bufs = [synthetic_batch(s, seed=500 + i, dtype=torch.float32).pin_memory() for i in range(n)]
        self.i = 0

    def __iter__(self) -> "PinnedBatches":
        return self

    def __next__(self) -> torch.Tensor:
        b = self.bufs[self.i % len(self.bufs)]
        self.i += 1
        return b


def run_e2e(s: BenchSetup, steps: int, warmup: int, sampler: Any = None) -> dict[str, Any]:
    from saelens_b200.config import LoggingConfig, SAETrainerConfig
    from saelens_b200.training.sae_trainer import SAETrainer

    rows_local = s.batch // s.world if s.world > 1 else s.batch
    local = BenchSetup(**{**s.__dict__, "batch": rows_local})
    sae = _materialise_local(_build_sae(s), s)
    if s.world > 1:
        sae._tp_group = dist.group.WORLD
    cfg = SAETrainerConfig(
        n_checkpoints=0, checkpoint_path=None, save_final_checkpoint=False, output_path=None,
        save_mse_every_n_steps=0, save_timing_every_n_steps=0, save_memory_every_n_steps=0,
        synchronize_timing=False, multi_sae_backward_order="forward", multi_sae_stats_sync_mode="immediate",
        multi_sae_stats_sync_interval=1, total_training_samples=(steps + warmup + 1) * s.batch,
        device=f"cuda:{torch.cuda.current_device()}", autocast=False, lr=s.lr, lr_end=s.lr / 10,
        lr_scheduler_name="constant", lr_warm_up_steps=0, adam_beta1=0.9, adam_beta2=0.999, lr_decay_steps=0,
        n_restart_cycles=1, train_batch_size_samples=s.batch, dead_feature_window=1000,
        feature_sampling_window=2000, logger=LoggingConfig(log_to_wandb=False), sae_engine="native",
        tp_exchange=s.tp_exchange,
    )
    from saelens_b200.training.prefetch import DevicePrefetcher

    data = DevicePrefetcher(PinnedBatches(local), device=cfg.device)
    trainer = SAETrainer(cfg, sae, data, tp_input_layout="row_sharded")
    trainer.fit_steps(warmup)
    torch.cuda.synchronize()
    _barrier(s.world)
    if sampler is not None:
        sampler.start()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record()
    trainer.fit_steps(steps, read_loss=True)
    t1.record()
    torch.cuda.synchronize()
    _barrier(s.world)
    clocks = sampler.stop() if sampler is not None else None
    ms = _max_over_ranks(t0.elapsed_time(t1) / steps, s.world)
    h2d = rows_local * s.d_in * 4  # fp32 rows from pinned host memory
    if hasattr(trainer.engine, "close"):
        trainer.engine.close()
    del trainer, sae, data
    _free()
    return {"ms_per_step": ms, "h2d_bytes": h2d, "d2h_bytes": 4, "clocks": clocks}


def parity_check(world: int, rank: int, d_in: int = 4096, d_sae: int = 16384, k: int = 128, batch: int = 2048,
                 steps: int = 3, lr: float = 1e-3, tp_exchange: str = "p2p") -> dict[str, Any]:
    """Tensor-parallel step against the single-GPU step on a small SAE, run before the timed region.

    Every rank builds the same full SAE (same seed) twice: one copy is latent-sharded and trained
    by the TP engine on this rank's rows of the batch, the other is trained whole by the single-GPU
    engine on the whole batch, on this rank's GPU.  Returns the largest relative loss difference
    and the largest difference of this rank's parameter shard (max over ranks), plus `ok`.  The
    dead-latent auxiliary loss runs on the second step."""
    from saelens_b200.models.topk import TopKTrainingSAE, TopKTrainingSAEConfig
    from saelens_b200.parallel.tp_engine import TPTopKEngine
    from saelens_b200.training.engine import FusedTopKEngine

    dev = torch.device("cuda", torch.cuda.current_device())

    def build() -> Any:
        torch.manual_seed(4321)
        sae = TopKTrainingSAE(TopKTrainingSAEConfig(d_in=d_in, d_sae=d_sae, k=k, device=str(dev)))
        with torch.no_grad():
            sae.b_enc.normal_(0, 0.01)
            sae.b_dec.normal_(0, 0.05)
        return sae

    g = torch.Generator(device="cpu").manual_seed(99)
    x = torch.randn(batch, d_in, generator=g)
    x = (x / x.norm(dim=-1, keepdim=True) * math.sqrt(d_in)).to(torch.bfloat16).to(dev)
    dead = (torch.arange(d_sae, device=dev) % 5) == 0
    n = d_sae // world
    rows = batch // world

    sae_tp = build()
    sae_tp.shard_weights(dist.group.WORLD)
    tp = TPTopKEngine(sae_tp, lr=lr, group=dist.group.WORLD, fused=tp_exchange == "p2p")
    tp_losses = [float(tp.step(x[rank * rows:(rank + 1) * rows].contiguous(), dead_mask=dead[rank * n:(rank + 1) * n],
                               run_aux=(i == 1)).loss) for i in range(steps)]
    torch.cuda.synchronize()
    tp.status.check("parity (tensor parallel)")
    one = FusedTopKEngine(build(), lr=lr)
    ref_losses = [float(one.step(x, dead_mask=dead, run_aux=(i == 1)).loss) for i in range(steps)]
    torch.cuda.synchronize()
    one.status.check("parity (single GPU)")
    loss_err = max(abs(a - b) / max(abs(b), 1e-12) for a, b in zip(tp_losses, ref_losses))
    sl = slice(rank * n, (rank + 1) * n)
    param_err = max((tp.p_dec - one.p_dec[sl]).abs().max().item(), (tp.p_enc - one.p_enc[sl]).abs().max().item(),
                    (tp.p_bdec - one.p_bdec).abs().max().item())
    if hasattr(tp, "close"):
        tp.close()
    del tp, one, sae_tp
    _free()
    loss_err = _max_over_ranks(loss_err, world)
    param_err = _max_over_ranks(param_err, world)
    # Adam moves every coordinate by at most lr per step, so parameters that differ by more
    # than a few lr after `steps` steps point at a wrong gradient, not at summation order.
    ok = loss_err <= 1e-3 and param_err <= 3 * steps * lr
    return {"max_rel_loss_err": loss_err, "max_param_err": param_err, "ok": bool(ok), "d_sae": d_sae,
            "batch": batch, "steps": steps}
