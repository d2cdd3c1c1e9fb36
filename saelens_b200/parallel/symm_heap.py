"""Symmetric peer memory for the NVLink kernels.

`SymmetricHeap` allocates one device slab per rank (`cudaMalloc`, zeroed), exports it with a
CUDA IPC handle, exchanges the handles over the process group once, and opens every peer's
slab.  Buffers are carved from the slab with a bump allocator; because every rank performs the
same sequence of `alloc` calls, a buffer sits at the same byte offset in every slab, and a
kernel reaches rank r's copy at `bases[r] + offset`.

Epoch flags and arrival counters used by the kernels live in the slab too.  They start at zero
and only grow (each use of a buffer set bumps its epoch), so they are never reset.

Creating a heap is a collective call: all ranks of `group` must construct it in the same order
with the same size.  The slab stays mapped until `close()` (also a collective).
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as dist

_ALIGN = 256


@dataclass(frozen=True)
class SlabBuffer:
    offset: int
    shape: tuple[int, ...]
    dtype: torch.dtype

    @property
    def nbytes(self) -> int:
        n = 1
        for s in self.shape:
            n *= s
        return n * torch.empty((), dtype=self.dtype).element_size()


class SymmetricHeap:
    def __init__(self, group: dist.ProcessGroup | None, nbytes: int, device: torch.device | int | None = None):
        from saelens_b200.ops import native

        self._nat = native()
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        if self.world > 8:
            raise ValueError("peer-memory kernels support at most 8 ranks (one NVSwitch domain)")
        if device is None:
            idx = torch.cuda.current_device()
        elif isinstance(device, int):
            idx = device
        else:
            d = torch.device(device)
            idx = d.index if d.index is not None else torch.cuda.current_device()
        self.device = torch.device("cuda", idx)
        self.nbytes = int((nbytes + _ALIGN - 1) // _ALIGN * _ALIGN)
        with torch.cuda.device(self.device):
            base, handle = self._nat.symm_alloc(self.nbytes)
        self.base = int(base)
        handles: list = [None] * self.world
        dist.all_gather_object(handles, (bytes(handle.numpy().tobytes()), self.nbytes), group=group)
        sizes = {h[1] for h in handles}
        if len(sizes) != 1:
            raise RuntimeError(f"symmetric heap sizes differ across ranks: {sorted(sizes)}")
        self.bases: list[int] = []
        self._opened: list[int] = []
        with torch.cuda.device(self.device):
            for r, (h, _) in enumerate(handles):
                if r == self.rank:
                    self.bases.append(self.base)
                else:
                    p = int(self._nat.symm_open(torch.frombuffer(bytearray(h), dtype=torch.uint8)))
                    self.bases.append(p)
                    self._opened.append(p)
        self._top = 0
        self.closed = False
        # every rank has mapped every slab before anyone writes into a peer's
        dist.barrier(group=group)

    # ------------------------------------------------------------------ allocation
    def alloc(self, shape: tuple[int, ...] | int, dtype: torch.dtype) -> SlabBuffer:
        shape = (shape,) if isinstance(shape, int) else tuple(int(s) for s in shape)
        buf = SlabBuffer(self._top, shape, dtype)
        end = self._top + buf.nbytes
        if end > self.nbytes:
            raise MemoryError(f"symmetric heap exhausted: need {end} bytes, have {self.nbytes}")
        self._top = (end + _ALIGN - 1) // _ALIGN * _ALIGN
        return buf

    def alloc_bytes(self, nbytes: int) -> int:
        return self.alloc((max(1, (int(nbytes) + 3) // 4),), torch.int32).offset

    def local(self, buf: SlabBuffer) -> torch.Tensor:
        """This rank's copy of `buf` as a tensor (a view into the slab)."""
        return self._nat.tensor_at(self.base + buf.offset, list(buf.shape), buf.dtype, self.device.index)

    def used(self) -> int:
        return self._top

    # ------------------------------------------------------------------ teardown
    def close(self) -> None:
        if self.closed:
            return
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        with torch.cuda.device(self.device):
            for p in self._opened:
                self._nat.symm_close(p)
            self._nat.symm_free(self.base)
        self._opened.clear()
        self.closed = True


def slab_bytes_needed(sizes: list[int]) -> int:
    """Total bytes for a sequence of allocations of the given sizes (with alignment)."""
    top = 0
    for n in sizes:
        top = (top + int(n) + _ALIGN - 1) // _ALIGN * _ALIGN
    return top
