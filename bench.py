"""Headline benchmark: SAE-training tokens/s of a tensor-parallel TopK SAE on N B200s.

Workload: the latent-sharded TopK SAE, d_in 4096, d_sae 1,048,576 (sharded N-way over latents),
k 128, batch 16384 tokens per step, bf16 compute with fp32 master weights and fp32 Adam
moments.  Inputs are synthetic activations ~N(0, 1) rescaled to norm sqrt(d_in); SAE weights
are random-init.  Total work is fixed as N grows (strong scaling).

`value` is the device-timed throughput: W untimed warm-up steps, then K steps bracketed by a
barrier and torch.cuda.synchronize(), timed with CUDA events and reduced with MAX over ranks.
`e2e` is the same metric through the public trainer API (`SAETrainer.fit_steps`), including
every step's pinned host->device copy of the input batch and a device->host read of the loss.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
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
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--d-in", type=int, default=4096)
    p.add_argument("--d-sae", type=int, default=1048576)
    p.add_argument("--k", type=int, default=128)
    p.add_argument("--batch", type=int, default=16384)
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--tp-exchange", choices=["p2p", "nccl"], default="p2p",
                   help="TP exchanges: fused NVLink peer-memory kernels (default) or NCCL collectives")
    return p.parse_args()


def _reference_arm(args: argparse.Namespace) -> None:
    reason = (
        "reference not installable offline: its build backend (poetry-core) and runtime deps "
        "(transformer_lens, datasets, wandb, simple_parsing, babe, nltk) are absent from the wheelhouse"
    )
    ref = os.path.join(ROOT, "baseline", "_ref", "sae_lens")
    if os.path.isdir(ref):
        reason = "baseline/_ref present but sae_lens cannot import without transformer_lens/datasets/wandb"
    rank = int(os.environ.get("RANK", "0"))
    if rank == 0:
        print(json.dumps({"impl": "reference", "unavailable": reason, "n_gpus": args.gpus}), flush=True)


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

    import torch
    import torch.distributed as dist

    from saelens_b200.training.bench_driver import BenchSetup, run_device_timed, run_e2e

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}; launch N>1 with torch.distributed.run")
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=600), device_id=torch.device("cuda", local))

    setup = BenchSetup(d_in=args.d_in, d_sae=args.d_sae, k=args.k, batch=args.batch, world=world, rank=rank,
                       tp_exchange=args.tp_exchange)
    sampler = ClockSampler(list(range(torch.cuda.device_count()))[:world] if world > 1 else [local]) if rank == 0 else None
    dev = run_device_timed(setup, args.steps, args.warmup, sampler)
    e2e = None if args.no_e2e else run_e2e(setup, args.steps, args.warmup)
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
        if e2e is not None:
            line["e2e"] = {"value": round(args.batch * 1000.0 / e2e["ms_per_step"], 1), "unit": "tokens/s",
                           "ms_per_step": round(e2e["ms_per_step"], 3),
                           "h2d_bytes_per_step": e2e["h2d_bytes"], "d2h_bytes_per_step": e2e["d2h_bytes"]}
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
