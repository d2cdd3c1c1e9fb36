"""Device-resident activation ring for streaming mode (producer and consumer GPUs disjoint).

The reference streams activations through a `/dev/shm` ring: producers copy chunks to host memory,
the consumer reads them back and H2D-copies them (sae_lens/training/shared_activation_buffer.py,
sae_lens/training/streaming_activation_provider.py:164-261).  Here the ring lives in the consumer
GPU's symmetric slab and never touches host memory:

* `write(x)` (producer): a bounded system-scope compare-and-swap claims a FREE slot in the
  consumer's state array over NVLink; one kernel stores the rows into that slot with P2P stores,
  normalising and casting to bf16 on the way; a release store marks the slot READY with its meta
  (rows, producer, sequence).
* `take(out, perm)` (consumer): claims a READY slot (scan from a rotating start, as the
  reference picks a random READY chunk), gathers its rows into `out` (optionally permuted: the
  provider's shuffle), and releases the slot as FREE.

Every device wait is bounded (`claim_timeout_ms`); the host retries until `timeout_s` and then
raises `TimeoutError`, so a stalled peer shows up as an exception, never as a hung GPU.  The
optional host header (`header_path`, a small file of int64 counters per rank: chunks written,
chunks taken, done flag) gives a supervisor a view of the ring without touching the GPUs.
"""

from __future__ import annotations

import time
from collections.abc import Callable
from pathlib import Path

import numpy as np
import torch
import torch.distributed as dist

from saelens_b200.parallel.symm_heap import SymmetricHeap, slab_bytes_needed

FREE, WRITING, READY, CONSUMING = 0, 1, 2, 3
_MODES = {"none": 0, "scale": 1, "unit_norm": 2}
HEADER_FIELDS = ("written", "taken", "done")


class HostRingHeader:
    """int64 [world, 3] counters in a file (memory-mapped); each rank writes only its own row."""

    def __init__(self, path: str | Path, world: int, rank: int, create: bool):
        self.path = Path(path)
        if create and not self.path.exists():
            np.zeros((world, len(HEADER_FIELDS)), dtype=np.int64).tofile(self.path)
        self.rank = rank
        self._mm = np.memmap(self.path, dtype=np.int64, mode="r+", shape=(world, len(HEADER_FIELDS)))

    def add(self, field: str, n: int = 1) -> None:
        self._mm[self.rank, HEADER_FIELDS.index(field)] += n
        self._mm.flush()

    def set(self, field: str, v: int) -> None:
        self._mm[self.rank, HEADER_FIELDS.index(field)] = v
        self._mm.flush()

    def snapshot(self) -> dict[str, list[int]]:
        arr = np.array(self._mm)
        return {f: arr[:, i].tolist() for i, f in enumerate(HEADER_FIELDS)}


class DeviceActivationRing:
    def __init__(self, group: dist.ProcessGroup | None, producer_ranks: list[int], consumer_rank: int,
                 n_slots: int, chunk_rows: int, d: int, normalize: str = "none", scale: float = 1.0,
                 header_path: str | Path | None = None, claim_timeout_ms: float = 1000.0):
        from saelens_b200.ops import native

        if normalize not in _MODES:
            raise ValueError(f"normalize must be one of {sorted(_MODES)}")
        if d % 8:
            raise ValueError("d must be a multiple of 8")
        self.nat = native()
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        if consumer_rank in producer_ranks:
            raise ValueError("the producer and consumer sets must be disjoint")
        self.producers, self.consumer = list(producer_ranks), int(consumer_rank)
        self.n_slots, self.chunk_rows, self.d = int(n_slots), int(chunk_rows), int(d)
        self.mode, self.scale = _MODES[normalize], float(scale)
        self.claim_timeout_ms = float(claim_timeout_ms)
        sizes = [n_slots * 4, n_slots * 16, 4 * self.world, n_slots * chunk_rows * d * 2]
        self.heap = SymmetricHeap(group, slab_bytes_needed(sizes) + 4096)
        self.state = self.heap.alloc(n_slots, torch.int32)
        self.meta = self.heap.alloc((n_slots, 4), torch.int32)
        self.done_flags = self.heap.alloc(self.world, torch.int32)
        self.data = self.heap.alloc((n_slots, chunk_rows, d), torch.bfloat16)
        dev = self.heap.device
        self.slot = torch.full((1,), -1, dtype=torch.int32, device=dev)
        self.seq = 0
        self.taken = 0
        self.header = None
        if header_path is not None:
            if self.rank == self.consumer:
                HostRingHeader(header_path, self.world, self.rank, create=True)
            dist.barrier(group=group)
            self.header = HostRingHeader(header_path, self.world, self.rank, create=False)

    # ------------------------------------------------------------------ helpers
    def _claim(self, owner: int, frm: int, to: int, start: int, timeout_s: float, what: str,
               stop_check: Callable[[], bool] | None = None) -> int | None:
        t0 = time.monotonic()
        while True:
            self.nat.ring_claim(self.heap.bases, self.rank, owner, self.state.offset, self.n_slots, frm, to, start,
                                self.claim_timeout_ms, self.slot)
            s = int(self.slot.item())
            if s >= 0:
                return s
            if stop_check is not None and stop_check():
                return None
            if time.monotonic() - t0 > timeout_s:
                raise TimeoutError(f"device ring: no {what} slot within {timeout_s:.1f} s")

    def local_state(self) -> torch.Tensor:
        """Slot states (consumer only)."""
        return self.heap.local(self.state)

    def local_meta(self) -> torch.Tensor:
        return self.heap.local(self.meta)

    # ------------------------------------------------------------------ producer
    def write(self, x: torch.Tensor, timeout_s: float = 60.0,
              stop_check: Callable[[], bool] | None = None) -> int | None:
        """Store `x` ([rows <= chunk_rows, d], fp32 or bf16, on this GPU) as one READY chunk.
        Returns the slot used.  Blocks (bounded waits, host retries) while the ring is full;
        returns None without writing when `stop_check()` turns true meanwhile."""
        if self.rank not in self.producers:
            raise RuntimeError(f"rank {self.rank} is not a producer of this ring")
        if x.dim() != 2 or x.shape[1] != self.d or x.shape[0] > self.chunk_rows:
            raise ValueError(f"chunk must be [<= {self.chunk_rows}, {self.d}]")
        p_idx = self.producers.index(self.rank)
        start = (self.seq * len(self.producers) + p_idx) % self.n_slots
        slot = self._claim(self.consumer, FREE, WRITING, start, timeout_s, "FREE", stop_check)
        if slot is None:
            return None
        self.nat.ring_write(x.contiguous(), self.heap.bases, self.rank, self.consumer, self.data.offset,
                            self.chunk_rows, self.slot, self.mode, self.scale)
        self.nat.ring_publish(self.heap.bases, self.rank, self.consumer, self.state.offset, self.meta.offset,
                              self.slot, int(x.shape[0]), p_idx, self.seq, READY)
        self.seq += 1
        if self.header is not None:
            self.header.add("written")
        return slot

    def producer_done(self) -> None:
        """Tell the consumer this producer will write no more chunks."""
        self.nat.p2p_signal(self.heap.bases, self.rank, self.done_flags.offset, self.rank, 1 << self.consumer, 1)
        torch.cuda.current_stream(self.heap.device).synchronize()
        if self.header is not None:
            self.header.set("done", 1)

    # ------------------------------------------------------------------ consumer
    def take(self, out: torch.Tensor | None = None, perm: torch.Tensor | None = None,
             timeout_s: float = 60.0, shuffle: torch.Generator | None = None) -> tuple[torch.Tensor, int]:
        """Claim a READY chunk, copy its rows into `out` ([rows, d] bf16 by default; `perm` int32
        picks the rows, or `shuffle` draws a permutation of the chunk's rows) and free the slot.
        Returns (out, rows in the chunk)."""
        if self.rank != self.consumer:
            raise RuntimeError(f"rank {self.rank} is not the consumer of this ring")
        start = (self.taken * 5 + 3) % self.n_slots
        slot = self._claim(self.rank, READY, CONSUMING, start, timeout_s, "READY")
        assert slot is not None
        rows = int(self.local_meta()[slot, 0].item())
        if perm is None and shuffle is not None:
            perm = torch.randperm(rows, device=self.heap.device, generator=shuffle, dtype=torch.int32)
        if out is None:
            out = torch.empty(rows, self.d, dtype=torch.bfloat16, device=self.heap.device)
        self.nat.ring_gather(self.heap.local(self.data), self.slot, perm, out)
        self.nat.ring_publish(self.heap.bases, self.rank, self.rank, self.state.offset, self.meta.offset,
                              self.slot, -1, 0, 0, FREE)
        self.taken += 1
        if self.header is not None:
            self.header.add("taken")
        return out, rows

    def producers_done(self) -> bool:
        """True once every producer called `producer_done` (consumer only)."""
        flags = self.heap.local(self.done_flags).cpu()
        return all(int(flags[r]) == 1 for r in self.producers)

    def ready_chunks(self) -> int:
        return int((self.local_state() == READY).sum().item())

    def close(self) -> None:
        self.heap.close()


__all__ = ["DeviceActivationRing", "HostRingHeader", "FREE", "WRITING", "READY", "CONSUMING"]
