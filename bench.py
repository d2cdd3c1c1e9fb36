"""Headline benchmark: SAE-training tokens/s of a tensor-parallel TopK SAE on N B200s.

Workload: the latent-sharded TopK SAE, d_in 4096, d_sae 1,048,576 (sharded N-way over latents),
k 128, batch 16384 tokens per step, bf16 compute with fp32 master weights and fp32 Adam
moments.  Inputs are synthetic activations ~N(0, 1) rescaled to norm sqrt(d_in); SAE weights
are random-init.  Total work is fixed as N grows (strong scaling).

`value` is the device-timed throughput: W untimed warm-up steps, then K steps bracketed by a
barrier and torch.cuda.synchronize(), timed with CUDA events and reduced with MAX over ranks.
`e2e` is the same metric through the public trainer API (`SAETrainer.fit_steps`), including
every step's pinned host->device copy of the fp32 input batch and a device->host read of the loss.
With N > 1 a small parity check (tensor-parallel step against the single-GPU step, d_sae 16384)
runs before the timed region; its result is printed and a failure exits non-zero.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference|eager]

`--impl reference` runs the reference package installed under baseline/_ref through its own
public API (`TopKTrainingSAE.shard_weights` + `SAETrainer._train_step`); when it cannot be
imported or run, the line says why.  `--impl eager` is this package's PyTorch restatement of the
reference's tensor-parallel math (all-gather of the pre-activations, dense top-k, dense decode,
all-reduce, torch.optim.Adam) on the same workload: an eager stand-in, not the reference.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

METRIC = "SAE-train tokens/sec (device-timed, max over ranks)"
PUBLISHED_VALUE = None  # the reference publishes no throughput number for this workload


def _parse() -> argparse.Namespace:
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=10)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", choices=["ours", "reference", "eager"], default="ours")
    p.add_argument("--d-in", type=int, default=4096)
    p.add_argument("--d-sae", type=int, default=1048576)
    p.add_argument("--k", type=int, default=128)
    p.add_argument("--batch", type=int, default=16384)
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--no-parity", action="store_true", help="skip the N>1 parity check before the timed region")
    p.add_argument("--tp-exchange", choices=["p2p", "nccl"], default="p2p",
                   help="TP exchanges: fused NVLink peer-memory kernels (default) or NCCL collectives")
    return p.parse_args()


def _dist_setup(args: argparse.Namespace):
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}; launch N>1 with torch.distributed.run")
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=600), device_id=torch.device("cuda", local))
    return world, rank, local


def _unavailable(impl: str, reason: str, args: argparse.Namespace, rank: int) -> None:
    if rank == 0:
        print(json.dumps({"impl": impl, "unavailable": reason, "n_gpus": args.gpus}), flush=True)


def _timed_steps(step, steps: int, warmup: int, world: int, sampler=None) -> tuple[float, dict | None]:
    """CUDA-event time per step of `step()` after `warmup` calls; max over ranks."""
    import torch
    import torch.distributed as dist

    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    if sampler is not None:
        sampler.start()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record()
    for _ in range(steps):
        step()
    t1.record()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clocks = sampler.stop() if sampler is not None else None
    ms = t0.elapsed_time(t1) / steps
    if world > 1:
        t = torch.tensor([ms], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    return ms, clocks


def _trainer_cfg_fields(args: argparse.Namespace, device: str) -> dict:
    return dict(n_checkpoints=0, checkpoint_path=None, save_final_checkpoint=False, output_path=None,
                save_mse_every_n_steps=0, save_timing_every_n_steps=0, save_memory_every_n_steps=0,
                synchronize_timing=False, multi_sae_backward_order="forward",
                multi_sae_stats_sync_mode="immediate", multi_sae_stats_sync_interval=1,
                total_training_samples=(args.steps + args.warmup + 1) * args.batch, device=device, autocast=False,
                lr=5e-5, lr_end=5e-6, lr_scheduler_name="constant", lr_warm_up_steps=0, adam_beta1=0.9,
                adam_beta2=0.999, lr_decay_steps=0, n_restart_cycles=1, train_batch_size_samples=args.batch,
                dead_feature_window=1000, feature_sampling_window=2000)


def _result_line(impl: str, args: argparse.Namespace, world: int, ms: float, clocks, parallelism: str) -> dict:
    value = args.batch * 1000.0 / ms
    return {"impl": impl, "metric": METRIC, "value": round(value, 1), "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 3), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None if PUBLISHED_VALUE is None else value / PUBLISHED_VALUE,
            "dtype": "bf16", "data": "synthetic: N(0,1) activations scaled to norm sqrt(d_in); random-init SAE",
            "config": {"model": f"TopK SAE d_in {args.d_in} d_sae {args.d_sae} k {args.k}",
                       "global_batch": args.batch, "seq_len": None, "parallelism": parallelism},
            "clocks": clocks}


def _reference_arm(args: argparse.Namespace) -> None:
    """The reference package from baseline/_ref, through its public API: `TopKTrainingSAE`
    latent-sharded with `shard_weights` over the whole job, every rank fed the full batch (the
    reference's TP input layout), `SAETrainer._train_step` timed per step
    (sae_lens/saes/topk_sae.py:448-674, sae_lens/training/sae_trainer.py:595-780)."""
    import traceback

    rank = int(os.environ.get("RANK", "0"))
    ref_root = os.path.join(ROOT, "baseline", "_ref")
    if not os.path.isdir(os.path.join(ref_root, "sae_lens")):
        _unavailable("reference", "baseline/_ref/sae_lens is absent: the offline pip install of the reference failed "
                     "(its build backend poetry-core is not in the wheelhouse)", args, rank)
        return
    sys.path.insert(0, ref_root)
    try:
        import sae_lens  # noqa: F401
        from sae_lens.config import LoggingConfig, SAETrainerConfig
        from sae_lens.saes.topk_sae import TopKTrainingSAE, TopKTrainingSAEConfig
        from sae_lens.training.sae_trainer import SAETrainer
    except Exception as e:  # the reason goes into the line verbatim
        _unavailable("reference", f"import sae_lens from baseline/_ref failed: {type(e).__name__}: {e}", args, rank)
        return
    import torch
    import torch.distributed as dist

    try:
        world, rank, local = _dist_setup(args)
        dev = f"cuda:{local}"
        torch.manual_seed(1234)
        sae = TopKTrainingSAE(TopKTrainingSAEConfig(d_in=args.d_in, d_sae=args.d_sae, k=args.k, dtype="bfloat16",
                                                    device=dev))
        if world > 1:
            sae.shard_weights(dist.group.WORLD)
        cfg = SAETrainerConfig(**_trainer_cfg_fields(args, dev), logger=LoggingConfig(log_to_wandb=False))
        trainer = SAETrainer(cfg, sae, data_provider=iter(()))
        g = torch.Generator(device=dev).manual_seed(100)
        x = torch.randn(args.batch, args.d_in, generator=g, device=dev)
        x = (x / x.norm(dim=-1, keepdim=True) * args.d_in ** 0.5).to(torch.bfloat16)

        def step() -> None:
            trainer._train_step(sae=trainer.sae, sae_in=x)
            trainer.n_training_steps += 1

        sampler = ClockSampler(list(range(world)) if world > 1 else [local]) if rank == 0 else None
        ms, clocks = _timed_steps(step, args.steps, args.warmup, world, sampler)
    except torch.OutOfMemoryError as e:
        _unavailable("reference", f"OOM: {str(e).splitlines()[0]}", args, rank)
        return
    except Exception as e:
        if rank == 0:
            traceback.print_exc()
        _unavailable("reference", f"reference step failed: {type(e).__name__}: {e}", args, rank)
        return
    if rank == 0:
        print(json.dumps(_result_line("reference", args, world, ms, clocks, f"tp{world}-nccl (reference)")),
              flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def _eager_arm(args: argparse.Namespace) -> None:
    """This package's PyTorch path with the reference's tensor-parallel math at the headline
    config: every rank gets the full batch, computes its latent shard's pre-activations, NCCL
    all-gathers them to [B, d_sae], takes the dense top-k, decodes its shard densely, all-reduces
    the reconstruction; autograd backward and torch.optim.Adam (`sae_engine="torch"`)."""
    import torch
    import torch.distributed as dist

    from saelens_b200.config import LoggingConfig, SAETrainerConfig
    from saelens_b200.models.topk import TopKTrainingSAE, TopKTrainingSAEConfig
    from saelens_b200.training.sae_trainer import SAETrainer

    world, rank, local = _dist_setup(args)
    dev = f"cuda:{local}"
    try:
        torch.manual_seed(1234)
        sae = TopKTrainingSAE(TopKTrainingSAEConfig(d_in=args.d_in, d_sae=args.d_sae, k=args.k, dtype="bfloat16",
                                                    device=dev))
        if world > 1:
            sae.shard_weights(dist.group.WORLD)
        cfg = SAETrainerConfig(**_trainer_cfg_fields(args, dev), logger=LoggingConfig(log_to_wandb=False),
                               sae_engine="torch")
        trainer = SAETrainer(cfg, sae, iter(()))
        g = torch.Generator(device=dev).manual_seed(100)
        x = torch.randn(args.batch, args.d_in, generator=g, device=dev)
        x = (x / x.norm(dim=-1, keepdim=True) * args.d_in ** 0.5).to(torch.bfloat16)

        def step() -> None:
            trainer._train_step(sae=trainer.sae, sae_in=x)
            trainer.n_training_steps += 1

        sampler = ClockSampler(list(range(world)) if world > 1 else [local]) if rank == 0 else None
        ms, clocks = _timed_steps(step, args.steps, args.warmup, world, sampler)
        ok = torch.tensor([1.0], device=dev)
    except torch.OutOfMemoryError as e:
        ms, clocks, ok = None, None, torch.tensor([0.0], device=dev)
        reason = f"OOM: {str(e).splitlines()[0]}"
    if world > 1:
        dist.all_reduce(ok, op=dist.ReduceOp.MIN)
    if ok.item() == 0.0:
        _unavailable("eager", reason if ms is None else "OOM on another rank", args, rank)
    elif rank == 0:
        print(json.dumps(_result_line("eager", args, world, ms, clocks, f"tp{world}-nccl (eager stand-in)")),
              flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


class ClockSampler:
    """Samples nvidia-smi clocks / throttle reasons in the background during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_indices: list[int]):
        self.gpus = set(gpu_indices)
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        self.proc: subprocess.Popen | None = None

    def start(self) -> None:
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=self.f, stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None

    def stop(self) -> dict:
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        self.f.flush()
        self.f.seek(0)
        mhz, maxes, reasons = [], [], set()
        for line in self.f.read().splitlines():
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 9 or not parts[0].isdigit() or int(parts[0]) not in self.gpus:
                continue
            try:
                sm, smax, pw = float(parts[1]), float(parts[2]), float(parts[3])
            except ValueError:
                continue
            if pw < 200:  # idle samples at the edges of the region
                continue
            mhz.append(sm)
            maxes.append(smax)
            for name, val in zip(("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"),
                                 parts[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        os.unlink(self.f.name)
        return {"sm_mhz": statistics.median(mhz) if mhz else None,
                "sm_max_mhz": max(maxes) if maxes else None, "reasons": sorted(reasons),
                "samples": len(mhz)}


def main() -> None:
    args = _parse()
    if args.impl == "reference":
        _reference_arm(args)
        return
    if args.impl == "eager":
        _eager_arm(args)
        return

    import torch
    import torch.distributed as dist

    from saelens_b200.training.bench_driver import BenchSetup, parity_check, run_device_timed, run_e2e

    world, rank, local = _dist_setup(args)
    parity = None
    if world > 1 and not args.no_parity:
        parity = parity_check(world, rank, tp_exchange=args.tp_exchange)
        if not parity["ok"]:
            if rank == 0:
                print(json.dumps({"metric": METRIC, "n_gpus": world, "parity": parity,
                                  "error": "tensor-parallel step differs from the single-GPU step"}), flush=True)
            dist.barrier()
            dist.destroy_process_group()
            sys.exit(3)
    setup = BenchSetup(d_in=args.d_in, d_sae=args.d_sae, k=args.k, batch=args.batch, world=world, rank=rank,
                       tp_exchange=args.tp_exchange)
    sampler = ClockSampler(list(range(torch.cuda.device_count()))[:world] if world > 1 else [local]) if rank == 0 else None
    dev = run_device_timed(setup, args.steps, args.warmup, sampler)
    e2e_sampler = ClockSampler(list(range(torch.cuda.device_count()))[:world] if world > 1 else [local]) \
        if rank == 0 else None
    e2e = None if args.no_e2e else run_e2e(setup, args.steps, args.warmup, e2e_sampler)
    if rank == 0:
        ms = dev["ms_per_step"]
        value = args.batch * 1000.0 / ms
        line = {
            "metric": METRIC, "value": round(value, 1), "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 3),
            "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None if PUBLISHED_VALUE is None else value / PUBLISHED_VALUE,
            "dtype": "bf16", "data": "synthetic: N(0,1) activations scaled to norm sqrt(d_in); random-init SAE",
            "config": {"model": f"TopK SAE d_in {args.d_in} d_sae {args.d_sae} k {args.k} (latent-sharded TP{world})",
                       "global_batch": args.batch, "seq_len": None, "parallelism": f"tp{world}" + (f"-{args.tp_exchange}" if world > 1 else ""),
                       "l2": "per-step working set (>17 GB of weights, 128 MB input) exceeds the 126 MB L2",
                       "optimizer": "Adam, fp32 master + fp32 moments, clip 1.0"},
            "clocks": dev.get("clocks"),
            "gpu_launches": dev["gpu_launches"],
        }
        if parity is not None:
            line["parity"] = {k: (round(v, 8) if isinstance(v, float) else v) for k, v in parity.items()}
        if e2e is not None:
            line["e2e"] = {"value": round(args.batch * 1000.0 / e2e["ms_per_step"], 1), "unit": "tokens/s",
                           "ms_per_step": round(e2e["ms_per_step"], 3),
                           "h2d_bytes_per_step": e2e["h2d_bytes"], "d2h_bytes_per_step": e2e["d2h_bytes"],
                           "input": "fp32 rows from pinned host memory, 8 distinct batches, copied on a side stream "
                                    "(DevicePrefetcher) overlapping the previous step; loss read back every step",
                           "clocks": e2e.get("clocks")}
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
