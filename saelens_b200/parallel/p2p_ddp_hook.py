"""DDP communication hook: every gradient bucket is averaged by the two-shot P2P all-reduce kernel
(ops/csrc/p2p.cu allreduce_kernel, 1/world scale fused) on a side CUDA stream.  DDP fires the hook
as soon as a bucket's gradients exist, so the NVLink reduction overlaps the rest of the backward
where DDP's NCCL all-reduce would run.  This serves every SAE that trains on the PyTorch path under
`sae_dp_mode="ddp"` (Standard/L1, Gated, JumpReLU, Matryoshka, transcoders); TopK and BatchTopK use
the native DDP engine instead.  Replaces the NCCL bucket all-reduce of the reference's DDP wrapping
(sae_lens/llm_sae_training_runner.py:449-485).

Peer memory: one data region (landing area + output area) sized for the largest bucket DDP can
form (bucket cap + the largest parameter), shared by every bucket, plus arrival counters and
flags per bucket shape.  Uses run one after another on the hook's stream.  A use ends on a rank
only after every owner has published its chunks, and an owner publishes only after reading its
landing area, so the next use may overwrite both areas.  Counters are per shape because their
targets grow by one epoch per use of that shape.
"""

from __future__ import annotations

import math
import os
from typing import Any

import torch
import torch.distributed as dist

from saelens_b200.parallel.symm_heap import SymmetricHeap, slab_bytes_needed

_DEFAULT_BUCKET_CAP_MB = 25.0


_MIN_RESERVE_BYTES = 256 << 20


def max_bucket_bytes(param_bytes: list[int], bucket_cap_mb: float | None) -> int:
    """Bytes of peer memory reserved for one bucket.  DDP usually closes a bucket once it exceeds
    the cap (at most cap + one parameter), but it may also put every parameter into one bucket,
    so the whole gradient is reserved when that is moderate; larger buckets fall back to NCCL."""
    cap = int((bucket_cap_mb if bucket_cap_mb is not None else _DEFAULT_BUCKET_CAP_MB) * 1024 * 1024)
    total = sum(param_bytes)
    return min(total, max(cap + max(param_bytes, default=0), _MIN_RESERVE_BYTES))


class P2PAllReduceHookState:
    def __init__(self, module: torch.nn.Module, group: dist.ProcessGroup | None,
                 bucket_cap_mb: float | None = None, counter_bytes: int = 16 << 20, max_ctas: int | None = None):
        from saelens_b200.ops import native
        from saelens_b200.ops.status import StatusWord

        self.nat = native()
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        params = [p for p in module.parameters() if p.requires_grad]
        if not params:
            raise ValueError("the module has no trainable parameters")
        self.device = params[0].device
        top = max_bucket_bytes([p.numel() * p.element_size() for p in params], bucket_cap_mb)
        # byte sizes of the largest bucket in either gradient width (chunk rounding differs)
        land = out = 0
        for esz in (2, 4):
            lb, _, ob, _ = self.nat.p2p_allreduce_sizes(math.ceil(top / esz), esz, self.world)
            land, out = max(land, lb), max(out, ob)
        self.land_bytes, self.out_bytes = land, out
        self.heap = SymmetricHeap(group, slab_bytes_needed([land, out, counter_bytes]) + 65536, self.device)
        self.land_off = self.heap.alloc_bytes(land)
        self.out_off = self.heap.alloc_bytes(out)
        self.areas: dict[tuple[int, torch.dtype], list[int]] = {}  # shape -> [cnt_off, flag_off, epoch]
        self.stream = torch.cuda.Stream(device=self.device)
        self.ticket = torch.zeros(1, dtype=torch.int32, device=self.device)
        self.status = StatusWord(self.device)
        self.calls = 0
        self.nccl_fallbacks = 0  # buckets larger than the reserved area (averaged by NCCL)
        # CTAs of the all-reduce kernel: it overlaps the backward, so it may be capped to leave SMs
        # to the compute (0 = as many as the transfer can use)
        if max_ctas is None:
            max_ctas = int(os.environ.get("SAELENS_B200_DDP_HOOK_CTAS", "0"))
        self.max_ctas = max(0, int(max_ctas))

    def _area(self, n: int, dtype: torch.dtype) -> list[int] | None:
        key = (n, dtype)
        a = self.areas.get(key)
        if a is None:
            esz = torch.empty((), dtype=dtype).element_size()
            land, cnt, out, flag = self.nat.p2p_allreduce_sizes(n, esz, self.world)
            if land > self.land_bytes or out > self.out_bytes:
                return None
            a = [self.heap.alloc_bytes(cnt), self.heap.alloc_bytes(flag), 0]
            self.areas[key] = a
        return a

    def reduce_(self, buf: torch.Tensor) -> torch.futures.Future:
        """Average `buf` over the group in place; the returned future completes on the hook's
        stream (consumers wait on it through the CUDA future semantics)."""
        n = buf.numel()
        if self._area(n, buf.dtype) is None:  # same decision on every rank: bucket shapes agree
            self.nccl_fallbacks += 1
            buf.div_(self.world)
            return dist.all_reduce(buf, group=self.group, async_op=True).get_future().then(lambda f: f.value()[0])
        cur = torch.cuda.current_stream(self.device)
        self.stream.wait_stream(cur)
        buf.record_stream(self.stream)
        with torch.cuda.stream(self.stream):
            a = self._area(n, buf.dtype)
            a[2] += 1
            # the kernel copies each averaged chunk back into the bucket as soon as it arrived
            self.nat.p2p_allreduce(buf, 1.0 / self.world, self.heap.bases, self.rank, self.land_off, a[0],
                                   self.out_off, a[1], a[2], self.ticket, self.status.tensor,
                                   max_ctas=self.max_ctas, x_out=buf)
            self.calls += 1
            fut: torch.futures.Future = torch.futures.Future(devices=[self.device])
            fut.set_result(buf)
        return fut

    def check(self, what: str = "ddp p2p all-reduce") -> None:
        self.status.check(what)

    def close(self) -> None:
        self.heap.close()


def p2p_allreduce_hook(state, bucket):  # noqa: ANN001, ANN201
    """`DistributedDataParallel.register_comm_hook(state, p2p_allreduce_hook)`.  No annotations:
    DDP checks them against `dist.GradBucket` / `Future[Tensor]` objects, and this module's
    postponed annotations would be strings."""
    return state.reduce_(bucket.buffer())


def p2p_hook_supported(module: torch.nn.Module, group: dist.ProcessGroup | None) -> bool:
    """CUDA parameters of fp32/bf16, at most 8 ranks (one NVSwitch domain), native ops built."""
    from saelens_b200 import ops

    params = [p for p in module.parameters() if p.requires_grad]
    if not params or not all(p.is_cuda and p.dtype in (torch.float32, torch.bfloat16) for p in params):
        return False
    world = dist.get_world_size(group)
    return 1 < world <= 8 and ops.available() and dist.get_backend(group) == "nccl"


def register_p2p_allreduce(ddp_module: Any, module: torch.nn.Module, group: dist.ProcessGroup | None,
                           bucket_cap_mb: float | None = None) -> P2PAllReduceHookState:
    state = P2PAllReduceHookState(module, group, bucket_cap_mb)
    ddp_module.register_comm_hook(state, p2p_allreduce_hook)
    return state


__all__ = ["P2PAllReduceHookState", "p2p_allreduce_hook", "p2p_hook_supported", "register_p2p_allreduce",
           "max_bucket_bytes"]
