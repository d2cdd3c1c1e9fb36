"""Measurement cases behind the committed profile summaries (run on a CUDA machine).

    python -m saelens_b200.perf_cases phases [--tp-exchange p2p|nccl] [--d-sae N]
        Per-phase CUDA-event times of the training step (one GPU, or several under
        torch.distributed.run: latent-sharded tensor parallel).
    python -m saelens_b200.perf_cases fused-case [--steps 2]
        Small fused tensor-parallel step with a world size of 1 (d_in 4096, d_sae 32768, k 128,
        batch 4096; about 2 GB on the device), the case used for ncu captures of the fused kernels.
    python -m saelens_b200.perf_cases gemm [--pair 0|1]
        Encoder GEMM numerics against fp32 and CUDA-event TFLOP/s on the benchmark shapes.
    python -m saelens_b200.perf_cases allreduce
        P2P two-shot all-reduce kernel vs NCCL all_reduce (bf16, sum) over sizes and chunk sizes,
        under torch.distributed.run; bus bandwidth = 2 (S-1)/S bytes / time, max time over ranks.
    python -m saelens_b200.perf_cases router [--rows 8192 --d 4096]
        Shard-routing transfer: rank 0 produces fp32 rows, the other ranks consume bf16 unit-norm
        rows; the fused P2P router vs NCCL send/recv with separate normalise + cast (max over ranks).
    python -m saelens_b200.perf_cases lm [--model llama-3-8b --stop 17 --batch 8 --ctx 1024]
        Producer LM forward up to the hooked layer on this package's kernels vs PyTorch ops.
    python -m saelens_b200.perf_cases ddp [--d-sae 131072 --k 64 --batch 8192 --steps 10]
        Data-parallel TopK step (replicated SAE, P2P gradient all-reduce) under
        torch.distributed.run: ms/step (max over ranks) and per-phase times.
    python -m saelens_b200.perf_cases fsdp-jumprelu [--d-in 3584 --d-sae 131072 --batch 4096]
        Sharded data-parallel JumpReLU at its dense init: native engine vs torch FSDP(FULL_SHARD).
    python -m saelens_b200.perf_cases attention [--batch 4 --ctx 2048 --heads 32 --kv-heads 8]
        Causal GQA prefill attention: tcgen05 kernel vs PyTorch SDPA, ms and TFLOP/s.
    python -m saelens_b200.perf_cases topology-switch --run-dir DIR --from-topo 1,2,4,1 --to-topo 1,4,4,1 ...
        Streaming run under the topology supervisor with one switch: timeline, downtime, tokens/s.
    python -m saelens_b200.perf_cases dense-step [--d-in 2304 --d-sae 65536 --batch 4096]
        Standard and Gated training steps: native dense engines vs the PyTorch (cuBLAS) path.
    python -m saelens_b200.perf_cases mp [--batch 4096 --d-in 768 --d-sae 24576 --iters 64]
        Matching-pursuit encode (forward, forward + backward): native kernels vs the PyTorch loop.
"""

from __future__ import annotations

import argparse
import json
import os
from datetime import timedelta
from typing import Any


def _init_dist() -> tuple[int, int, int]:
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if not dist.is_initialized():
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        os.environ.setdefault("MASTER_PORT", "29533")
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    return world, rank, local


def phases(args: argparse.Namespace) -> None:
    os.environ["SAELENS_B200_PHASE_TIMING"] = "1"
    import torch
    import torch.distributed as dist

    from saelens_b200.training.bench_driver import BenchSetup, _make_engine, synthetic_batch

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = 0
    if world > 1:
        world, rank, _ = _init_dist()
    s = BenchSetup(d_in=args.d_in, d_sae=args.d_sae, k=args.k, batch=args.batch, world=world, rank=rank,
                   tp_exchange=args.tp_exchange, arch=args.arch)
    eng = _make_engine(s)
    x = synthetic_batch(BenchSetup(**{**s.__dict__, "batch": args.batch // world}), 1 + rank, device="cuda")
    for _ in range(3):
        eng.step(x)
    eng.phase_times_ms()
    n = 5
    for _ in range(n):
        eng.step(x)
    t = eng.phase_times_ms()
    print(rank, args.tp_exchange if world > 1 else "single",
          json.dumps({k: round(v / n, 3) for k, v in t.items()}), "total_ms", round(sum(t.values()) / n, 2),
          "tokens_per_s", round(args.batch / (sum(t.values()) / n) * 1e3, 1), flush=True)
    if args.arch == "batchtopk":
        print(rank, "truncated_rows", int(eng.batch_truncated.item()), "topk_threshold",
              float(eng.sae.topk_threshold), flush=True)
    eng.status.check()
    eng.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def tpdp(args: argparse.Namespace) -> None:
    """Tensor x data parallel step: TP groups of `--tp` consecutive ranks, DP groups across them.
    Each DP replica trains on `--batch` rows per step (split over its TP ranks); tokens/s counts
    all replicas.  Device time from CUDA events over the steps, max over ranks."""
    os.environ["SAELENS_B200_PHASE_TIMING"] = "1"
    import torch
    import torch.distributed as dist

    from saelens_b200.parallel.tp_engine import TPTopKEngine
    from saelens_b200.training.bench_driver import BenchSetup, _build_sae, _materialise_local, synthetic_batch

    world, rank, _ = _init_dist()
    tp_size = args.tp
    if world % tp_size:
        raise SystemExit(f"world {world} is not a multiple of tp {tp_size}")
    dp_size = world // tp_size
    tp_groups = [dist.new_group(list(range(d * tp_size, (d + 1) * tp_size))) for d in range(dp_size)]
    dp_groups = [dist.new_group(list(range(t, world, tp_size))) for t in range(tp_size)]
    tp_rank, dp_rank = rank % tp_size, rank // tp_size
    s = BenchSetup(d_in=args.d_in, d_sae=args.d_sae, k=args.k, batch=args.batch, world=tp_size, rank=tp_rank,
                   arch=args.arch)
    sae = _materialise_local(_build_sae(s), s)
    eng = TPTopKEngine(sae, lr=s.lr, group=tp_groups[dp_rank], fused=True, dp_group=dp_groups[tp_rank])
    x = synthetic_batch(BenchSetup(**{**s.__dict__, "batch": args.batch // tp_size}), 1 + rank, device="cuda")
    for _ in range(3):
        eng.step(x)
    eng.phase_times_ms()
    torch.cuda.synchronize()
    dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        eng.step(x)
    e1.record()
    torch.cuda.synchronize()
    t = torch.tensor([e0.elapsed_time(e1) / args.steps], device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ph = eng.phase_times_ms()
    ms = float(t.item())
    if rank == 0:
        print(json.dumps({"tp": tp_size, "dp": dp_size, "arch": args.arch, "d_in": args.d_in, "d_sae": args.d_sae,
                          "k": args.k, "batch_per_replica": args.batch, "ms_per_step": round(ms, 3),
                          "tokens_per_s": round(args.batch * dp_size / ms * 1e3, 1),
                          "phases_ms": {k: round(v / args.steps, 3) for k, v in ph.items()}}), flush=True)
    eng.status.check()
    eng.close()
    dist.barrier()
    dist.destroy_process_group()


def fused_case(args: argparse.Namespace) -> None:
    import torch
    import torch.distributed as dist

    _init_dist()
    from saelens_b200.parallel.tp_engine import TPTopKEngine
    from saelens_b200.training.bench_driver import BenchSetup, _build_sae, _materialise_local, synthetic_batch

    s = BenchSetup(d_in=4096, d_sae=32768, k=128, batch=4096, world=1, rank=0)
    sae = _materialise_local(_build_sae(s), s)
    eng = TPTopKEngine(sae, lr=5e-5, group=dist.group.WORLD, fused=True)
    x = synthetic_batch(s, 1, device="cuda")
    for _ in range(args.steps):
        eng.step(x)
    torch.cuda.synchronize()
    eng.status.check()
    print(json.dumps({"ok": True, "loss": float(eng.last_loss)}))
    eng.close()
    dist.destroy_process_group()


def gemm(args: argparse.Namespace) -> None:
    os.environ["SAELENS_B200_GEMM_PAIR"] = str(args.pair)
    import torch

    from saelens_b200.ops import native
    from saelens_b200.ops.status import StatusWord

    nat = native()
    st = StatusWord("cuda")
    torch.manual_seed(0)
    print("pair" if args.pair else "single", flush=True)
    for M, N, K, relu, timing in ((256, 256, 64, False, False), (512, 1024, 256, False, False),
                                  (300, 512, 128, True, False), (4096, 32768, 4096, False, True),
                                  (4096, 262144, 4096, False, True)):
        A = (torch.randn(M, K, device="cuda") * 0.5).to(torch.bfloat16)
        B = (torch.randn(N, K, device="cuda") * 0.5).to(torch.bfloat16)
        bias = torch.randn(N, device="cuda")
        scale = torch.rand(N, device="cuda") + 0.5
        out = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
        cm = torch.empty(M, N // 32, dtype=torch.bfloat16, device="cuda")
        nat.gemm_tn_bf16(A, B, bias, scale, relu, out, cm, st.tensor, 0)
        torch.cuda.synchronize()
        ref = (A.float() @ B.float().T + bias) * scale
        if relu:
            ref = ref.relu()
        err = ((out.float() - ref).abs().max() / ref.abs().max()).item()
        line = f"M={M} N={N} K={K} status={st.code()} rel_max_err={err:.2e}"
        if timing and st.code() == 0:
            for _ in range(3):
                nat.gemm_tn_bf16(A, B, bias, scale, relu, out, cm, st.tensor, 0)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(10):
                nat.gemm_tn_bf16(A, B, bias, scale, relu, out, cm, st.tensor, 0)
            e1.record()
            torch.cuda.synchronize()
            ms = e0.elapsed_time(e1) / 10
            line += f" ms={ms:.3f} TFLOPs={2 * M * N * K / ms / 1e9:.1f}"
        print(line, flush=True)
        st.check("gemm")


def gemm_step(args: argparse.Namespace) -> None:
    """Encoder GEMM of the headline step (one 4096-row chunk: 4096 x d_sae x 4096) under the power
    cap: the CTA-pair and single-CTA tcgen05 kernels with the full epilogue (bias, ||W_dec|| scale,
    bf16 store, 32-column and tile maxima) and without stores, against cuBLAS (torch.matmul, bf16
    output).  CUDA-event ms over `reps` back-to-back launches, TFLOP/s and the median SM clock."""
    import subprocess
    import tempfile

    import torch

    from saelens_b200.ops import native
    from saelens_b200.ops.status import StatusWord

    nat = native()
    st = StatusWord("cuda")
    M, N, K = args.m, args.n, args.k
    torch.manual_seed(0)
    A = (torch.randn(M, K, device="cuda") * 0.5).to(torch.bfloat16)
    B = (torch.randn(N, K, device="cuda") * 0.02).to(torch.bfloat16)
    bias = torch.randn(N, device="cuda")
    scale = torch.rand(N, device="cuda") + 0.5
    out = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
    cm = torch.empty(M, N // 32, dtype=torch.bfloat16, device="cuda")
    tm = torch.empty(M, N // 256, dtype=torch.bfloat16, device="cuda")

    def ours(full: bool):
        return lambda: nat.gemm_tn_bf16(A, B, bias if full else None, scale if full else None, False,
                                        out if full else None, cm if full else None, st.tensor, 0,
                                        tmax=tm if full else None)

    def cublas():
        torch.matmul(A, B.T, out=out)

    def timed(fn):
        for _ in range(2):
            fn()
        torch.cuda.synchronize()
        log = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        smi = subprocess.Popen(["nvidia-smi", "-i", str(torch.cuda.current_device()), "--query-gpu=clocks.sm,power.draw",
                                "--format=csv,noheader,nounits", "-lms", "100"], stdout=log, stderr=subprocess.DEVNULL)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.reps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        smi.terminate()
        smi.wait()
        log.seek(0)
        mhz = sorted(float(x.split(",")[0]) for x in log.read().splitlines() if x.strip() and float(x.split(",")[1]) > 300)
        return e0.elapsed_time(e1) / args.reps, (mhz[len(mhz) // 2] if mhz else None)

    res = {}
    # pair_full stores H with TMA tile stores from a staging tile; pair_full_rowstores with the
    # per-thread row stores (SAELENS_B200_GEMM_TMA_STORE=0)
    for name, pair, tma, fn in (("pair_full", "1", "1", ours(True)), ("pair_full_rowstores", "1", "0", ours(True)),
                                ("pair_nostore", "1", "1", ours(False)), ("single_full", "0", "1", ours(True)),
                                ("cublas", "1", "1", cublas)):
        os.environ["SAELENS_B200_GEMM_PAIR"] = pair
        os.environ["SAELENS_B200_GEMM_TMA_STORE"] = tma
        ms, mhz = timed(fn)
        st.check(name)
        res[name] = {"ms": round(ms, 3), "tflops": round(2 * M * N * K / ms / 1e9, 1), "sm_mhz": mhz}
    print(json.dumps({"M": M, "N": N, "K": K, **res}), flush=True)


def ddp(args: argparse.Namespace) -> None:
    os.environ["SAELENS_B200_PHASE_TIMING"] = "1"
    import torch
    import torch.distributed as dist

    from saelens_b200.models.topk import TopKTrainingSAE, TopKTrainingSAEConfig
    from saelens_b200.parallel.ddp_engine import DDPTopKEngine
    from saelens_b200.training.bench_driver import BenchSetup, synthetic_batch

    world, rank, local = _init_dist()
    torch.manual_seed(1234)
    d_in = getattr(args, "d_in", 4096)
    sae = TopKTrainingSAE(TopKTrainingSAEConfig(d_in=d_in, d_sae=args.d_sae, k=args.k, device=f"cuda:{local}"))
    if getattr(args, "engine", "ddp") == "fsdp":
        from saelens_b200.parallel.fsdp_engine import FSDPTopKEngine

        eng = FSDPTopKEngine(sae, lr=5e-5, group=dist.group.WORLD)
    else:
        eng = DDPTopKEngine(sae, lr=5e-5, group=dist.group.WORLD, segments=args.segments)
    s = BenchSetup(d_in=d_in, d_sae=args.d_sae, k=args.k, batch=args.batch, world=1, rank=rank)
    xs = [synthetic_batch(s, 10 * i + rank, device="cuda") for i in range(2)]
    for i in range(3):
        eng.step(xs[i % 2])
    eng.phase_times_ms()
    torch.cuda.synchronize()
    dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(args.steps):
        eng.step(xs[i % 2])
    e1.record()
    torch.cuda.synchronize()
    ms = torch.tensor([e0.elapsed_time(e1) / args.steps], device="cuda")
    dist.all_reduce(ms, op=dist.ReduceOp.MAX)
    t = eng.phase_times_ms()
    eng.status.check()
    if rank == 0:
        print(json.dumps({"engine": getattr(args, "engine", "ddp"), "world": world, "d_in": d_in,
                          "d_sae": args.d_sae, "k": args.k, "batch_per_gpu": args.batch,
                          "ms_per_step": round(float(ms.item()), 3),
                          "tokens_per_s": round(args.batch * world * 1000.0 / float(ms.item()), 1),
                          "phases_ms": {k: round(v / args.steps, 3) for k, v in t.items()}}), flush=True)
    eng.close()
    dist.barrier()
    dist.destroy_process_group()


def ddp_hook(args: argparse.Namespace) -> None:
    """PyTorch-path SAE under torch DDP (by default JumpReLU, d_in 3584, d_sae 131072, 4096 rows per GPU):
    gradient buckets averaged by the P2P all-reduce hook vs DDP's NCCL all-reduce.  Device time
    from CUDA events over the steps, max over ranks."""
    import torch
    import torch.distributed as dist
    from torch.nn.parallel import DistributedDataParallel as DDP

    from saelens_b200.models.jumprelu import JumpReLUTrainingSAE, JumpReLUTrainingSAEConfig
    from saelens_b200.models.sae import TrainStepInput
    from saelens_b200.models.standard import StandardTrainingSAE, StandardTrainingSAEConfig
    from saelens_b200.parallel.p2p_ddp_hook import register_p2p_allreduce
    from saelens_b200.training.bench_driver import BenchSetup, synthetic_batch

    world, rank, local = _init_dist()
    dev = f"cuda:{local}"
    x = synthetic_batch(BenchSetup(d_in=args.d_in, d_sae=args.d_sae, k=1, batch=args.batch, world=1, rank=rank),
                        1 + rank, device="cuda").float()
    res = {}
    for mode in ("p2p", "nccl"):
        torch.manual_seed(1234)
        if args.arch == "jumprelu":
            sae = JumpReLUTrainingSAE(JumpReLUTrainingSAEConfig(
                d_in=args.d_in, d_sae=args.d_sae, jumprelu_init_threshold=0.001, jumprelu_bandwidth=0.001,
                l0_coefficient=1.0, device=dev))
            coef = {"l0": 1.0}
        else:
            sae = StandardTrainingSAE(StandardTrainingSAEConfig(d_in=args.d_in, d_sae=args.d_sae, device=dev))
            coef = {"l1": 5.0}
        ddp = DDP(sae, device_ids=[local])
        state = register_p2p_allreduce(ddp, sae, dist.group.WORLD) if mode == "p2p" else None
        opt = torch.optim.Adam(sae.parameters(), lr=5e-5)

        def step(i: int) -> None:
            with torch.autocast("cuda", dtype=torch.bfloat16):
                out = ddp(TrainStepInput(sae_in=x, coefficients=coef, dead_neuron_mask=None, n_training_steps=i))
            out.loss.backward()
            opt.step()
            opt.zero_grad(set_to_none=False)

        for i in range(3):
            step(i)
        torch.cuda.synchronize()
        dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for i in range(args.steps):
            step(i)
        e1.record()
        torch.cuda.synchronize()
        t = torch.tensor([e0.elapsed_time(e1) / args.steps], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        res[mode] = round(float(t.item()), 3)
        if state is not None:
            state.check()
            res["p2p_nccl_fallbacks"] = state.nccl_fallbacks
            state.close()
        del ddp, opt, sae
        torch.cuda.empty_cache()
    if rank == 0:
        print(json.dumps({"world": world, "arch": args.arch, "d_in": args.d_in, "d_sae": args.d_sae,
                          "batch_per_gpu": args.batch, "ms_per_step": res,
                          "tokens_per_s": {m: round(args.batch * world / res[m] * 1e3, 1) for m in ("p2p", "nccl")},
                          "precision": "fp32 params, bf16 autocast"}), flush=True)
    dist.barrier()
    dist.destroy_process_group()


def ring(args: argparse.Namespace) -> None:
    """Streaming transport throughput, rank 0 producer -> rank 1 consumer: chunks of fp32 rows
    normalised to norm sqrt(d) and cast to bf16, through the device ring (P2P stores into the
    consumer GPU) and through the /dev/shm ring (D2H, shared memory, pinned H2D).  Consumer-side
    CUDA events around the whole stream of chunks; GB/s counts the bf16 rows delivered."""
    import math
    import tempfile

    import torch
    import torch.distributed as dist

    from saelens_b200.parallel.device_ring import DeviceActivationRing
    from saelens_b200.training.shared_activation_buffer import SharedActivationBuffer
    from saelens_b200.training.streaming_activation_provider import StreamingActivationProvider

    world, rank, _ = _init_dist()
    rows, d, n = args.rows, args.d, args.chunks
    x = torch.randn(rows, d, device="cuda")
    res = {}
    # device ring
    ringd = DeviceActivationRing(dist.group.WORLD, [0], 1, n_slots=4, chunk_rows=rows, d=d, normalize="unit_norm",
                                 scale=math.sqrt(d))
    dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if rank == 0:
        for _ in range(n):
            ringd.write(x)
        torch.cuda.synchronize()
    else:
        out = torch.empty(rows, d, dtype=torch.bfloat16, device="cuda")
        ringd.take(out=out)  # first chunk: warm-up
        e0.record()
        for _ in range(n - 1):
            ringd.take(out=out)
        e1.record()
        torch.cuda.synchronize()
        res["device_ms_per_chunk"] = e0.elapsed_time(e1) / (n - 1)
    dist.barrier()
    ringd.close()
    # host ring (/dev/shm): the reference's transport
    import shutil

    need = 4 * rows * d * 2 + (1 << 20)
    base = "/dev/shm" if os.path.isdir("/dev/shm") and shutil.disk_usage("/dev/shm").free > need \
        else tempfile.gettempdir()
    name_t = torch.tensor([os.getpid()], device="cuda")
    dist.broadcast(name_t, src=0)
    name = f"perf_ring_{int(name_t.item())}"
    if rank == 0:
        buf = SharedActivationBuffer(name, 4, rows, d, num_producers=1, target_chunks=n, create=True, base_dir=base)
    dist.barrier()
    if rank == 1:
        buf = SharedActivationBuffer(name, 4, rows, d, num_producers=1, target_chunks=n, base_dir=base)
    dist.barrier()
    if rank == 0:
        for _ in range(n):
            got = buf.allocate_write_chunk()
            if got is None:
                break
            y = (x / x.norm(dim=-1, keepdim=True) * math.sqrt(d)).to(torch.bfloat16).cpu()
            buf.write_chunk(got[0], y, rows)
            buf.mark_ready(got[0])
        buf.signal_done()
    else:
        prov = StreamingActivationProvider(buf, rows, 1, "cuda", d_model=d, dtype=torch.bfloat16, shuffle=False,
                                           random_chunks=False)
        next(prov)
        e0.record()
        for _ in range(n - 1):
            next(prov)
        e1.record()
        torch.cuda.synchronize()
        res["host_ms_per_chunk"] = e0.elapsed_time(e1) / (n - 1)
    dist.barrier()
    buf.close()
    if rank == 0:
        buf.unlink()
    if rank == 1:
        gb = rows * d * 2 / 1e9
        print(json.dumps({"rows": rows, "d": d, "chunks": n, **{k: round(v, 3) for k, v in res.items()},
                          "device_GBs": round(gb / res["device_ms_per_chunk"] * 1e3, 1),
                          "host_GBs": round(gb / res["host_ms_per_chunk"] * 1e3, 1)}), flush=True)
    dist.barrier()
    dist.destroy_process_group()


def allreduce(args: argparse.Namespace) -> None:
    import torch
    import torch.distributed as dist

    from saelens_b200.ops import native
    from saelens_b200.ops.status import StatusWord
    from saelens_b200.parallel.symm_heap import SlabBuffer, SymmetricHeap

    world, rank, _ = _init_dist()
    nat = native()
    st = StatusWord("cuda")
    tk = torch.zeros(1, dtype=torch.int32, device="cuda")
    sizes = [1 << 20, 16 << 20, 256 << 20, 1 << 30]  # bytes
    chunks = [4096, 16384, 65536]
    need = max(sum(nat.p2p_allreduce_sizes(n // 2, 2, world, c)) for n in sizes for c in chunks) + (1 << 20)
    heap = SymmetricHeap(dist.group.WORLD, need)

    def timed(fn, reps: int) -> float:
        fn()
        torch.cuda.synchronize()
        dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        t = torch.tensor([e0.elapsed_time(e1) / reps], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    rows = []
    for nbytes in sizes:
        n = nbytes // 2
        x = torch.randn(n, device="cuda").to(torch.bfloat16)
        reps = 20 if nbytes <= (16 << 20) else 5
        y = x.clone()
        ms = timed(lambda: dist.all_reduce(y), reps)
        bus = 2 * (world - 1) / world * nbytes / ms / 1e6
        rows.append({"bytes": nbytes, "impl": "nccl", "ms": round(ms, 4), "busbw_GBs": round(bus, 1)})
        for c in chunks:
            land, cnt, out, flag = nat.p2p_allreduce_sizes(n, 2, world, c)
            heap._top = 0
            o_land, o_cnt = heap.alloc_bytes(land), heap.alloc_bytes(cnt)
            o_out, o_flag = heap.alloc_bytes(out), heap.alloc_bytes(flag)
            ep = [0]

            def run() -> None:
                ep[0] += 1
                nat.p2p_allreduce(x, 1.0, heap.bases, rank, o_land, o_cnt, o_out, o_flag, ep[0], tk, st.tensor,
                                  -1, c)

            # fresh counters for this layout: zero them on every rank, then agree before use
            torch.cuda.synchronize()
            heap.local(SlabBuffer(o_cnt, (cnt // 4,), torch.int32)).zero_()
            heap.local(SlabBuffer(o_flag, (flag // 4,), torch.int32)).zero_()
            torch.cuda.synchronize()
            dist.barrier()
            ms = timed(run, reps)
            st.check("allreduce")
            bus = 2 * (world - 1) / world * nbytes / ms / 1e6
            rows.append({"bytes": nbytes, "impl": f"p2p chunk {c}", "ms": round(ms, 4), "busbw_GBs": round(bus, 1)})
        del x, y
    if rank == 0:
        for r in rows:
            print(json.dumps(r), flush=True)
    heap.close()
    dist.destroy_process_group()


def router(args: argparse.Namespace) -> None:
    import math

    import torch
    import torch.distributed as dist

    from saelens_b200.parallel.row_router import P2PRowRouter
    from saelens_b200.parallel.shard_routing import compute_routing_table

    world, rank, _ = _init_dist()
    producers, consumers = [0], list(range(1, world)) if world > 1 else [0]
    rows, d = args.rows, args.d
    scale = math.sqrt(d)
    x = torch.randn(rows, d, device="cuda")
    r = P2PRowRouter(dist.group.WORLD, producers, consumers, rows, d, normalize="unit_norm", scale=scale)
    routes = compute_routing_table(1, len(consumers), rows)

    def p2p_step() -> None:
        if rank in producers:
            r.send(x)
        if rank in consumers:
            r.recv()
            r.release()

    recv_bufs = {c: torch.empty(rt.n_rows, d, dtype=torch.bfloat16, device="cuda")
                 for c, rt in zip(consumers, routes)}

    def nccl_step() -> None:
        ops = []
        if rank in producers:
            y = (x / x.norm(dim=-1, keepdim=True) * scale).to(torch.bfloat16)
            for c, rt in zip(consumers, routes):
                ops.append(dist.P2POp(dist.isend, y[rt.row_start : rt.row_end].contiguous(), c))
        if rank in consumers:
            ops.append(dist.P2POp(dist.irecv, recv_bufs[rank], producers[0]))
        if ops:
            for w in dist.batch_isend_irecv(ops):
                w.wait()

    def timed(fn, reps: int = 20) -> float:
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        t = torch.tensor([e0.elapsed_time(e1) / reps], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    ms_p2p = timed(p2p_step)
    r.status.check("router")
    ms_nccl = float("nan") if args.no_nccl else timed(nccl_step)
    bytes_out = rows * d * 2
    if rank == 0:
        print(json.dumps({"world": world, "rows": rows, "d": d, "p2p_ms": round(ms_p2p, 4),
                          "nccl_ms": round(ms_nccl, 4), "p2p_GBs": round(bytes_out / ms_p2p / 1e6, 1),
                          "nccl_GBs": round(bytes_out / ms_nccl / 1e6, 1),
                          "note": "bytes = bf16 rows leaving the producer; fp32 input read once"}), flush=True)
    r.close()
    dist.destroy_process_group()


def lm(args: argparse.Namespace) -> None:
    """Producer LM forward up to the hooked layer (activation capture), one GPU: CUDA-event ms per
    forward on this package's kernels against the same model on PyTorch ops (F.linear / cuBLAS,
    scaled_dot_product_attention / cuDNN or flash, torch norms), plus achieved TFLOP/s."""
    import torch

    from saelens_b200.models.lm import transformer as T
    from saelens_b200.models.lm.transformer import HookedLM, preset_config

    torch.cuda.set_device(0)
    cfg = preset_config(args.model, n_layers=args.stop, dtype="bfloat16")
    torch.manual_seed(0)
    model = HookedLM(cfg, device="cuda")
    tokens = torch.randint(0, cfg.d_vocab, (args.batch, args.ctx), device="cuda")
    H, KV, dh, d = cfg.n_heads, cfg.n_key_value_heads, cfg.d_head, cfg.d_model
    per_tok = 2 * (d * H * dh + 2 * d * KV * dh + H * dh * d + (3 if cfg.gated_mlp else 2) * d * cfg.d_mlp)
    attn = 2 * 2 * (args.ctx + 1) / 2 * H * dh  # causal QK^T and PV per token (mean over positions)
    flops = args.batch * args.ctx * args.stop * (per_tok + attn)
    res = {"model": args.model, "layers_run": args.stop, "batch": args.batch, "ctx": args.ctx}
    arms = (("native", True),) if args.native_only else (("native", True), ("torch", False))
    for name, native in arms:
        T.FORCE_TORCH = not native
        with torch.no_grad():
            for _ in range(2):
                model(tokens, stop_at_layer=args.stop)
            torch.cuda.synchronize()
            t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            t0.record()
            for _ in range(args.reps):
                out = model(tokens, stop_at_layer=args.stop)
            t1.record()
            torch.cuda.synchronize()
        ms = t0.elapsed_time(t1) / args.reps
        res[name] = {"ms": round(ms, 3), "tokens_per_s": round(args.batch * args.ctx / ms * 1e3, 1),
                     "tflops": round(flops / ms / 1e9, 1)}
        res[name + "_out_norm"] = float(out.float().norm())
    T.FORCE_TORCH = False
    print(json.dumps(res), flush=True)


def fsdp_jumprelu(args: argparse.Namespace) -> None:
    """Sharded data-parallel JumpReLU at the dense init (threshold 0.001, bandwidth 0.001, L0
    coefficient 1; default d_in 3584, d_sae 131072, 4096 rows per GPU): the native engine
    (parameter all-gather fused into the encoder GEMM, reduce-scatter fused into the gradient GEMMs,
    sharded Adam) against torch FSDP(FULL_SHARD) over NCCL with bf16 autocast and torch Adam, the
    reference's wrapping (sae_lens/llm_sae_training_runner.py:449-463).  Device time from CUDA events
    over the steps, max over ranks."""
    import torch
    import torch.distributed as dist

    from saelens_b200.models.jumprelu import JumpReLUTrainingSAE, JumpReLUTrainingSAEConfig
    from saelens_b200.models.sae import TrainStepInput
    from saelens_b200.parallel.fsdp_jumprelu_engine import FSDPJumpReLUEngine
    from saelens_b200.training.bench_driver import BenchSetup, synthetic_batch

    world, rank, local = _init_dist()
    dev = f"cuda:{local}"
    x = synthetic_batch(BenchSetup(d_in=args.d_in, d_sae=args.d_sae, k=1, batch=args.batch, world=1, rank=rank),
                        1 + rank, device="cuda")

    def build() -> JumpReLUTrainingSAE:
        torch.manual_seed(1234)
        return JumpReLUTrainingSAE(JumpReLUTrainingSAEConfig(
            d_in=args.d_in, d_sae=args.d_sae, jumprelu_init_threshold=0.001, jumprelu_bandwidth=0.001,
            l0_coefficient=1.0, device=dev))

    def timed(step) -> float:
        for i in range(3):
            step(i)
        torch.cuda.synchronize()
        dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for i in range(args.steps):
            step(i)
        e1.record()
        torch.cuda.synchronize()
        t = torch.tensor([e0.elapsed_time(e1) / args.steps], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return round(float(t.item()), 3)

    res: dict[str, float] = {}
    os.environ["SAELENS_B200_PHASE_TIMING"] = "1"  # per-phase CUDA events of the native engine
    eng = FSDPJumpReLUEngine(build(), lr=5e-5, group=dist.group.WORLD)
    res["native"] = timed(lambda i: eng.step(x))
    eng.status.check()
    # the events also ran during the warm-up steps: phase means over warm-up + timed steps
    phases = {k: round(v / (3 + args.steps), 3) for k, v in eng.phase_times_ms().items()}
    eng.close()
    del eng
    torch.cuda.empty_cache()
    if not args.no_torch:
        from torch.distributed.fsdp import FullyShardedDataParallel as FSDP
        from torch.distributed.fsdp import ShardingStrategy

        sae = build()
        fs = FSDP(sae, sharding_strategy=ShardingStrategy.FULL_SHARD, device_id=torch.device(dev),
                  use_orig_params=True)
        opt = torch.optim.Adam(fs.parameters(), lr=5e-5)
        xf = x.float()

        def step(i: int) -> None:
            with torch.autocast("cuda", dtype=torch.bfloat16):
                out = fs(TrainStepInput(sae_in=xf, coefficients={"l0": 1.0}, dead_neuron_mask=None,
                                        n_training_steps=i))
            out.loss.backward()
            fs.clip_grad_norm_(1.0)
            opt.step()
            opt.zero_grad(set_to_none=False)

        res["torch_fsdp"] = timed(step)
        del fs, opt, sae
        torch.cuda.empty_cache()
    if rank == 0:
        print(json.dumps({"world": world, "arch": "jumprelu", "d_in": args.d_in, "d_sae": args.d_sae,
                          "batch_per_gpu": args.batch, "ms_per_step": res,
                          "tokens_per_s": {m: round(args.batch * world / v * 1e3, 1) for m, v in res.items()},
                          "native_phases_ms": phases,
                          "native": "bf16 compute, fp32 master + Adam state, sharded",
                          "torch_fsdp": "fp32 params, bf16 autocast, FULL_SHARD over NCCL"}), flush=True)
    dist.barrier()
    dist.destroy_process_group()


def attention_case(args: argparse.Namespace) -> None:
    """Causal GQA prefill attention, one GPU: the tcgen05 kernel (`ops.attention`) against PyTorch
    scaled_dot_product_attention (flash / cuDNN) on the same bf16 [B, S, H, D] inputs.  CUDA-event
    ms per call after warm-up; TFLOP/s counts the causal half of QK^T and PV (2 B H S^2 D)."""
    import torch
    import torch.nn.functional as F

    from saelens_b200 import ops

    B, S, H, KV, D = args.batch, args.ctx, args.heads, args.kv_heads, args.head_dim
    g = torch.Generator(device="cuda").manual_seed(0)
    q = torch.randn(B, S, H, D, device="cuda", generator=g).to(torch.bfloat16)
    k = torch.randn(B, S, KV, D, device="cuda", generator=g).to(torch.bfloat16)
    v = torch.randn(B, S, KV, D, device="cuda", generator=g).to(torch.bfloat16)
    out = torch.empty_like(q)
    st = ops.StatusWord("cuda")
    scale = D ** -0.5

    def ours() -> None:
        ops.attention(q, k, v, scale, out=out, status=st)

    qt, kt, vt = q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2)

    def sdpa() -> None:
        F.scaled_dot_product_attention(qt, kt, vt, is_causal=True, scale=scale, enable_gqa=True)

    def timed(fn) -> float:
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.reps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / args.reps

    flops = 2.0 * B * H * S * S * D  # causal: half of 4 B H S^2 D
    res = {}
    for w in ("8", "4"):  # softmax warps: half rows / whole rows (the default, timed last)
        os.environ["SAELENS_B200_ATTN_WARPS"] = w
        res[f"ours{w}_ms"] = round(timed(ours), 4)
        st.check("attention")
    if not args.no_sdpa:
        res["sdpa_ms"] = round(timed(sdpa), 4)
    res.update({k2.replace("_ms", "_tflops"): round(flops / v2 / 1e9, 1) for k2, v2 in list(res.items())})
    ref = F.scaled_dot_product_attention(qt.float(), kt.float(), vt.float(), is_causal=True, scale=scale,
                                         enable_gqa=True).transpose(1, 2)
    ours()
    res["max_abs_err_vs_fp32"] = float((out.float() - ref).abs().max())
    print(json.dumps({"batch": B, "ctx": S, "heads": H, "kv_heads": KV, "head_dim": D, **res}), flush=True)


def topology_switch(args: argparse.Namespace) -> None:
    """Topology switch of a streaming run under the supervisor (scripts/topology_supervisor.py:366-517
    in the reference): the worker group starts with `--from-topo`, a switch to `--to-topo` is
    requested after `--steps-before` trainer steps, the supervisor quiesces (producer dataset
    positions, SAE checkpoint, acks), relaunches from the quiesce checkpoint and the run completes.
    Prints the supervisor's event timeline, the switch downtime (arrival time of the first trainer
    step after the relaunch minus that of the last one before the quiesce) and the trainer's tokens/s
    before and after (its own elapsed-time records).  Topologies are vllm_tp,vllm_dp,sae_tp,sae_dp;
    every other `--field value` goes to the workers."""
    import math
    import signal
    import subprocess
    import threading
    import time
    from pathlib import Path

    from saelens_b200.runners.topology_supervisor import (
        TopologySupervisor,
        build_torchrun_cmd,
        request_topology_switch,
    )
    from saelens_b200.runners.worker import parse as parse_worker
    from saelens_b200.topology_control import BufferParams, TopologySpec

    def topo(spec: str) -> TopologySpec:
        a = [int(v) for v in spec.split(",")]
        return TopologySpec(*a)

    run_dir = Path(args.run_dir)
    ring_dir = Path(args.ring_dir)
    run_dir.mkdir(parents=True, exist_ok=True)
    ring_dir.mkdir(parents=True, exist_ok=True)
    worker_cfg = list(args.worker_args)
    if not any(a in ("--output_path", "--output-path") for a in worker_cfg):
        worker_cfg += ["--output_path", str(run_dir / "out")]
    worker_cfg += ["--streaming_buffer_dir", str(ring_dir)]
    _, wcfg = parse_worker(worker_cfg)
    out = Path(wcfg.output_path)
    params = BufferParams(wcfg.streaming_num_chunks, wcfg.streaming_chunk_size_tokens, wcfg.sae.d_in,
                          "float32" if wcfg.dtype in ("float32", "torch.float32") else "bfloat16")
    target = math.ceil(wcfg.training_tokens / wcfg.streaming_chunk_size_tokens)
    procs: list[subprocess.Popen] = []

    def launch(state: Any) -> subprocess.Popen:
        cmd = build_torchrun_cmd("-m saelens_b200.runners.worker", state.topology, run_dir, worker_cfg)
        if state.checkpoint_path:
            cmd += ["--resume-from-checkpoint", state.checkpoint_path]
        log = open(run_dir / f"workers_{state.epoch}.log", "w")
        p = subprocess.Popen(cmd, stdout=log, stderr=subprocess.STDOUT, start_new_session=True)
        procs.append(p)
        return p

    sup = TopologySupervisor(run_dir, topo(args.from_topo), launch, buffer_name=f"sb_switch_{os.getpid()}",
                             buffer_params=params, target_chunks=target, buffer_base_dir=str(ring_dir), poll_s=0.5,
                             exit_timeout_s=120.0, ack_timeout_s=300.0)
    result: dict[str, int] = {}
    th = threading.Thread(target=lambda: result.setdefault("rc", sup.run()), daemon=True)
    th.start()
    hist = out / "timing_history.jsonl"
    seen: list[tuple[float, dict]] = []  # (arrival wall time, record)

    def poll() -> None:
        if hist.exists():
            for ln in hist.read_text().splitlines()[len(seen):]:
                if ln.strip():
                    seen.append((time.time(), json.loads(ln)))

    t0, requested, n_before = time.time(), None, 0
    try:
        while th.is_alive():
            poll()
            if requested is None and len(seen) >= args.steps_before:
                request_topology_switch(run_dir, topo(args.to_topo))
                requested = time.time()
            if time.time() - t0 > args.max_s:
                raise SystemExit(f"topology switch run exceeded {args.max_s} s")
            time.sleep(0.1)
    finally:
        for p in procs:  # the worker groups this case started, by their own process-group ids
            if p.poll() is None:
                os.killpg(p.pid, signal.SIGTERM)
    poll()
    events = [json.loads(x) for x in (run_dir / "topology_switch_log.jsonl").read_text().splitlines()]
    t_quiesce = next((e["time"] for e in events if e["event"] == "quiesce_signaled"), None)
    relaunch = [e["time"] for e in events if e["event"] == "workers_launched"][1:2]
    before = [(w, r) for w, r in seen if t_quiesce is None or w < t_quiesce]
    after = [(w, r) for w, r in seen if relaunch and w > relaunch[0]]
    n_before = len(before)

    def rate(recs: list[tuple[float, dict]]) -> float | None:
        recs = recs[3:]  # skip the warm-up steps of a (re)launch
        if len(recs) < 2:
            return None
        (_, a), (_, b) = recs[0], recs[-1]
        dt = b["elapsed_s"] - a["elapsed_s"]
        return round((b["n_training_samples"] - a["n_training_samples"]) / dt, 1) if dt > 0 else None

    last_before = max((w for w, _ in seen if t_quiesce is not None and w < t_quiesce), default=None)
    first_after = after[0][0] if after else None
    print(json.dumps({
        "from": args.from_topo, "to": args.to_topo, "rc": result.get("rc"),
        "events": [{"event": e["event"], "t_s": round(e["time"] - events[0]["time"], 2)} for e in events],
        "steps_before_switch": n_before, "steps_after_switch": len(after),
        "downtime_s": round(first_after - last_before, 2) if (first_after and last_before) else None,
        "tokens_per_s_before": rate(before), "tokens_per_s_after": rate(after),
    }), flush=True)


def dense_step(args: argparse.Namespace) -> None:
    """Standard (ReLU + L1) and Gated SAE training steps, one GPU: the native dense engines
    (tcgen05 GEMMs with fused epilogues, row-fused Adam) against the PyTorch path on the same
    shapes (fp32 parameters, bf16 autocast, cuBLAS GEMMs through autograd, torch Adam, clip 1.0).
    CUDA-event ms per step after 3 warm-up steps."""
    import torch

    from saelens_b200.models.gated import GatedTrainingSAE, GatedTrainingSAEConfig
    from saelens_b200.models.sae import TrainStepInput
    from saelens_b200.models.standard import StandardTrainingSAE, StandardTrainingSAEConfig
    from saelens_b200.training.bench_driver import BenchSetup, synthetic_batch
    from saelens_b200.training.dense_engine import GatedEngine, StandardEngine

    x = synthetic_batch(BenchSetup(d_in=args.d_in, d_sae=args.d_sae, k=1, batch=args.batch, world=1, rank=0), 1,
                        device="cuda")
    xf = x.float()

    def timed(step) -> float:
        for i in range(3):
            step(i)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for i in range(args.steps):
            step(i)
        e1.record()
        torch.cuda.synchronize()
        return round(e0.elapsed_time(e1) / args.steps, 3)

    res: dict[str, dict[str, float]] = {}
    for arch, cls, cfg_cls, eng_cls, coef in (
            ("standard", StandardTrainingSAE, StandardTrainingSAEConfig, StandardEngine, {"l1": 5.0}),
            ("gated", GatedTrainingSAE, GatedTrainingSAEConfig, GatedEngine, {"l1": 5.0})):
        torch.manual_seed(0)
        eng = eng_cls(cls(cfg_cls(d_in=args.d_in, d_sae=args.d_sae, l1_coefficient=5.0, device="cuda")), lr=5e-5)
        native = timed(lambda i: eng.step(x))
        eng.status.check(arch)
        del eng
        torch.cuda.empty_cache()
        torch.manual_seed(0)
        sae = cls(cfg_cls(d_in=args.d_in, d_sae=args.d_sae, l1_coefficient=5.0, device="cuda"))
        opt = torch.optim.Adam(sae.parameters(), lr=5e-5)

        def step(i: int) -> None:
            with torch.autocast("cuda", dtype=torch.bfloat16):
                out = sae.training_forward_pass(TrainStepInput(sae_in=xf, coefficients=coef, dead_neuron_mask=None,
                                                               n_training_steps=i))
            out.loss.backward()
            sae.clip_grad_norm_(1.0)
            opt.step()
            opt.zero_grad(set_to_none=False)

        torch_ms = timed(step)
        del sae, opt
        torch.cuda.empty_cache()
        res[arch] = {"native_ms": native, "torch_ms": torch_ms, "speedup": round(torch_ms / native, 2),
                     "native_tokens_per_s": round(args.batch / native * 1e3, 1)}
    print(json.dumps({"d_in": args.d_in, "d_sae": args.d_sae, "batch": args.batch, **res}), flush=True)


def mp_case(args: argparse.Namespace) -> None:
    """Matching-pursuit encode, one GPU: the native path (tcgen05 score GEMM with fused row argmax
    + fused per-row update; `ops.mp`) against the PyTorch loop of the reference's iteration, on
    the same fp32 inputs, for a forward alone and a forward + backward of sum(codes * g).  Inputs
    are sparse combinations of a random unit-norm dictionary plus noise; the run stops by the
    reference's rules (duplicate support, residual threshold) or at --iters.  CUDA-event ms per
    call after one warm-up call; also the iterations run and the mean L0."""
    import torch

    from saelens_b200.models.matching_pursuit import _encode_matching_pursuit_torch
    from saelens_b200.ops import mp

    B, D, N = args.batch, args.d_in, args.d_sae
    g = torch.Generator(device="cuda").manual_seed(0)
    W = torch.randn(N, D, device="cuda", generator=g)
    W = W / W.norm(dim=1, keepdim=True)
    cols = torch.randint(0, N, (B, args.active), device="cuda", generator=g)
    codes = torch.zeros(B, N, device="cuda").scatter_(1, cols, torch.rand(B, args.active, device="cuda",
                                                                         generator=g) + 0.5)
    x = codes @ W + args.noise * torch.randn(B, D, device="cuda", generator=g)
    del codes
    g_out = torch.randn(B, N, device="cuda", generator=g)
    it = args.iters

    def native_fwd():
        with torch.no_grad():
            return mp.encode_matching_pursuit(x, W, args.thresh, it, True)

    def torch_fwd():
        with torch.no_grad():
            return _encode_matching_pursuit_torch(x, W, args.thresh, it, True)

    def native_fb():
        xr, Wr = x.detach().requires_grad_(True), W.detach().requires_grad_(True)
        (mp.encode_matching_pursuit(xr, Wr, args.thresh, it, True) * g_out).sum().backward()

    def torch_fb():
        xr, Wr = x.detach().requires_grad_(True), W.detach().requires_grad_(True)
        (_encode_matching_pursuit_torch(xr, Wr, args.thresh, it, True) * g_out).sum().backward()

    def timed(fn) -> float:
        fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.reps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / args.reps

    _, _, idx, _ = mp.trace_matching_pursuit(x, W, args.thresh, it, True)
    acts = native_fwd()
    res = {"iterations": int(idx.shape[0]), "mean_l0": round(float((acts != 0).sum(1).float().mean()), 2),
           "rel_residual": round(float(((x - acts @ W).norm(dim=1) / x.norm(dim=1)).mean()), 4)}
    del acts
    res["native_fwd_ms"] = round(timed(native_fwd), 3)
    res["native_fwd_bwd_ms"] = round(timed(native_fb), 3)
    if not args.no_torch:
        res["torch_fwd_ms"] = round(timed(torch_fwd), 3)
        res["torch_fwd_bwd_ms"] = round(timed(torch_fb), 3)
        res["speedup_fwd"] = round(res["torch_fwd_ms"] / res["native_fwd_ms"], 2)
        res["speedup_fwd_bwd"] = round(res["torch_fwd_bwd_ms"] / res["native_fwd_bwd_ms"], 2)
    gemm_flops = 2.0 * B * D * N * res["iterations"]
    res["score_gemm_tflops_equiv"] = round(gemm_flops / res["native_fwd_ms"] / 1e9, 1)
    print(json.dumps({"batch": B, "d_in": D, "d_sae": N, **res}), flush=True)


def main() -> None:
    p = argparse.ArgumentParser(prog="python -m saelens_b200.perf_cases")
    sub = p.add_subparsers(dest="cmd", required=True)
    a = sub.add_parser("phases")
    a.add_argument("--tp-exchange", choices=["p2p", "nccl"], default="p2p")
    a.add_argument("--d-sae", type=int, default=1048576)
    a.add_argument("--d-in", type=int, default=4096)
    a.add_argument("--k", type=int, default=128)
    a.add_argument("--batch", type=int, default=16384, help="rows per step over the whole TP group")
    a.add_argument("--arch", choices=["topk", "batchtopk"], default="topk")
    b = sub.add_parser("fused-case")
    b.add_argument("--steps", type=int, default=2)
    c = sub.add_parser("gemm")
    c.add_argument("--pair", type=int, choices=[0, 1], default=1)
    d = sub.add_parser("ddp")
    d.add_argument("--d-in", type=int, default=4096)
    d.add_argument("--d-sae", type=int, default=131072)
    d.add_argument("--k", type=int, default=64)
    d.add_argument("--batch", type=int, default=8192)
    d.add_argument("--steps", type=int, default=10)
    d.add_argument("--segments", type=int, default=4)
    fs = sub.add_parser("fsdp", help="sharded data parallel engine (latent-sharded optimizer state)")
    fs.add_argument("--d-in", type=int, default=3584)
    fs.add_argument("--d-sae", type=int, default=131072)
    fs.add_argument("--k", type=int, default=64)
    fs.add_argument("--batch", type=int, default=4096)
    fs.add_argument("--steps", type=int, default=10)
    fs.set_defaults(engine="fsdp", segments=1)
    td = sub.add_parser("tpdp")
    td.add_argument("--tp", type=int, default=4)
    td.add_argument("--arch", choices=["topk", "batchtopk"], default="batchtopk")
    td.add_argument("--d-in", type=int, default=5120)
    td.add_argument("--d-sae", type=int, default=327680)
    td.add_argument("--k", type=int, default=64)
    td.add_argument("--batch", type=int, default=8192, help="rows per step and data-parallel replica")
    td.add_argument("--steps", type=int, default=10)
    dh = sub.add_parser("ddp-hook", help="PyTorch-path SAE under DDP: P2P all-reduce hook vs NCCL")
    dh.add_argument("--arch", choices=["jumprelu", "standard"], default="jumprelu")
    dh.add_argument("--d-in", type=int, default=3584)
    dh.add_argument("--d-sae", type=int, default=131072)
    dh.add_argument("--batch", type=int, default=4096)
    dh.add_argument("--steps", type=int, default=10)
    rg = sub.add_parser("ring", help="streaming transport throughput: device ring vs /dev/shm ring (2 ranks)")
    rg.add_argument("--rows", type=int, default=8192)
    rg.add_argument("--d", type=int, default=4096)
    rg.add_argument("--chunks", type=int, default=24)
    sub.add_parser("allreduce")
    fj = sub.add_parser("fsdp-jumprelu", help="sharded data-parallel JumpReLU: native engine vs torch FSDP")
    fj.add_argument("--d-in", type=int, default=3584)
    fj.add_argument("--d-sae", type=int, default=131072)
    fj.add_argument("--batch", type=int, default=4096)
    fj.add_argument("--steps", type=int, default=10)
    fj.add_argument("--no-torch", action="store_true", help="skip the torch FSDP comparison")
    at = sub.add_parser("attention", help="causal GQA prefill attention: tcgen05 kernel vs PyTorch SDPA")
    at.add_argument("--batch", type=int, default=4)
    at.add_argument("--ctx", type=int, default=2048)
    at.add_argument("--heads", type=int, default=32)
    at.add_argument("--kv-heads", type=int, default=8)
    at.add_argument("--head-dim", type=int, default=128)
    at.add_argument("--reps", type=int, default=10)
    at.add_argument("--no-sdpa", action="store_true", help="time only the tcgen05 kernel (profiling runs)")
    ts = sub.add_parser("topology-switch", help="streaming run under the supervisor with one topology switch")
    ts.add_argument("--run-dir", required=True)
    ts.add_argument("--ring-dir", default="/dev/shm")
    ts.add_argument("--from-topo", default="1,1,1,1", help="vllm_tp,vllm_dp,sae_tp,sae_dp")
    ts.add_argument("--to-topo", default="1,2,1,1")
    ts.add_argument("--steps-before", type=int, default=20)
    ts.add_argument("--max-s", type=float, default=900.0)
    dsp = sub.add_parser("dense-step", help="Standard / Gated steps: native dense engines vs the PyTorch path")
    dsp.add_argument("--d-in", type=int, default=2304)
    dsp.add_argument("--d-sae", type=int, default=65536)
    dsp.add_argument("--batch", type=int, default=4096)
    dsp.add_argument("--steps", type=int, default=10)
    rt = sub.add_parser("router")
    rt.add_argument("--rows", type=int, default=8192)
    rt.add_argument("--d", type=int, default=4096)
    rt.add_argument("--no-nccl", action="store_true", help="skip the NCCL comparison (1-GPU profiling runs)")
    gs = sub.add_parser("gemm-step", help="headline encoder GEMM chunk: ours (pair / single, with / without "
                                         "stores) vs cuBLAS under the power cap")
    gs.add_argument("--m", type=int, default=4096)
    gs.add_argument("--n", type=int, default=1048576)
    gs.add_argument("--k", type=int, default=4096)
    gs.add_argument("--reps", type=int, default=10)
    lmp = sub.add_parser("lm", help="producer LM forward to the hooked layer: native kernels vs PyTorch ops")
    lmp.add_argument("--model", default="llama-3-8b")
    lmp.add_argument("--stop", type=int, default=17, help="blocks run (hook layer + 1)")
    lmp.add_argument("--batch", type=int, default=8)
    lmp.add_argument("--ctx", type=int, default=1024)
    lmp.add_argument("--reps", type=int, default=5)
    lmp.add_argument("--native-only", action="store_true", help="skip the PyTorch-ops arm (launch lists)")
    mpc = sub.add_parser("mp", help="matching-pursuit encode: native kernels vs the PyTorch loop")
    mpc.add_argument("--batch", type=int, default=4096)
    mpc.add_argument("--d-in", type=int, default=768)
    mpc.add_argument("--d-sae", type=int, default=24576)
    mpc.add_argument("--active", type=int, default=16, help="dictionary atoms per synthetic row")
    mpc.add_argument("--noise", type=float, default=0.02)
    mpc.add_argument("--thresh", type=float, default=0.01)
    mpc.add_argument("--iters", type=int, default=64)
    mpc.add_argument("--reps", type=int, default=3)
    mpc.add_argument("--no-torch", action="store_true")
    args, rest = p.parse_known_args()
    if args.cmd == "topology-switch":
        args.worker_args = rest
    elif rest:
        p.error(f"unrecognized arguments: {' '.join(rest)}")
    {"gemm-step": gemm_step, "lm": lm, "phases": phases, "fused-case": fused_case, "gemm": gemm, "ddp": ddp, "allreduce": allreduce, "router": router,
     "tpdp": tpdp, "fsdp": ddp, "ddp-hook": ddp_hook, "ring": ring, "fsdp-jumprelu": fsdp_jumprelu,
     "attention": attention_case, "topology-switch": topology_switch, "dense-step": dense_step,
     "mp": mp_case}[args.cmd](args)


if __name__ == "__main__":
    main()
