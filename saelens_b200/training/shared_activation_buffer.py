"""Host shared-memory ring of activation chunks between producer and trainer processes.

Producers claim a FREE slot (bounded by a global chunk quota), write `chunk_size_tokens x d_model`
rows into it and mark it READY; trainers claim READY slots (random order), read them and release
them back to FREE.  State machine FREE -> WRITING -> READY -> CONSUMING -> FREE, the transitions
serialised by an `fcntl` lock, the data itself read and written without the lock (a slot is owned
exclusively while WRITING or CONSUMING).  Behaviour of sae_lens/training/shared_activation_buffer.py.

Layout (this package's own, two memory-mapped files plus a lock file in `base_dir`):
  {name}.ctl   int64 words: header[16] then per-slot [state, valid_rows, producer_id, seq_no]
               header: 0 magic, 1 version, 2 num_slots, 3 chunk_tokens, 4 d_model, 5 dtype code
               (0 bf16, 1 fp32), 6 num_producers, 7 done_count, 8 target_chunks, 9 next_claim_seq
  {name}.dat   raw rows [num_slots, chunk_tokens, d_model] (bf16 bit patterns or fp32)
  {name}.lock  empty file for fcntl.flock
`reset_for_restart` lets a supervisor recycle abandoned WRITING slots between worker launches.

On a CUDA process `register_for_device_copies()` page-locks the data mapping for the copy engines
(cudaHostRegister): a producer then copies device activations straight into its slot and a trainer
copies claimed slots straight to the device, with no pageable host copy in between.  The mapping
is MAP_SHARED, so the processes see each other's rows without an msync; the data file is flushed
only on close.
"""

from __future__ import annotations

import fcntl
import random as _random
import shutil
import time
from collections.abc import Callable, Iterator
from contextlib import contextmanager
from enum import IntEnum
from pathlib import Path

import numpy as np
import torch

_MAGIC = 0x53414542  # "SAEB"
_VERSION = 1
_HDR = 16
_SLOT_WORDS = 4


class ChunkState(IntEnum):
    FREE = 0
    WRITING = 1
    READY = 2
    CONSUMING = 3


_DTYPE_CODE = {torch.bfloat16: 0, torch.float32: 1}
_CODE_DTYPE = {0: torch.bfloat16, 1: torch.float32}
_CODE_NP = {0: np.uint16, 1: np.float32}


class SharedActivationBuffer:
    def __init__(self, name: str, num_chunks: int, chunk_size_tokens: int, d_model: int, num_producers: int,
                 target_chunks: int = 0, create: bool = False, base_dir: str = "/dev/shm",
                 dtype: torch.dtype = torch.bfloat16) -> None:
        self._name = name
        self._n = num_chunks
        self._T = chunk_size_tokens
        self._D = d_model
        base = Path(base_dir)
        ctl, dat, lock = base / f"{name}.ctl", base / f"{name}.dat", base / f"{name}.lock"
        self.paths = (ctl, dat, lock)
        if create:
            if dtype not in _DTYPE_CODE:
                raise ValueError(f"SharedActivationBuffer supports bfloat16 or float32, got {dtype}")
            code = _DTYPE_CODE[dtype]
            nbytes = num_chunks * chunk_size_tokens * d_model * (2 if code == 0 else 4)
            if shutil.disk_usage(str(base)).free < nbytes + (1 << 20):
                raise RuntimeError(f"Insufficient space in {base_dir} for {nbytes} bytes of activations")
            c = np.memmap(str(ctl), dtype=np.int64, mode="w+", shape=(_HDR + _SLOT_WORDS * num_chunks,))
            c[:] = 0
            c[:10] = [_MAGIC, _VERSION, num_chunks, chunk_size_tokens, d_model, code, num_producers, 0,
                      target_chunks, 0]
            c.flush()
            d = np.memmap(str(dat), dtype=_CODE_NP[code], mode="w+",
                          shape=(num_chunks, chunk_size_tokens, d_model))
            d.flush()
            del c, d
            lock.touch(exist_ok=True)
        self._ctl = np.memmap(str(ctl), dtype=np.int64, mode="r+")
        if int(self._ctl[0]) != _MAGIC or int(self._ctl[1]) != _VERSION:
            raise ValueError(f"{ctl} is not a saelens_b200 activation ring")
        if (int(self._ctl[2]), int(self._ctl[3]), int(self._ctl[4])) != (num_chunks, chunk_size_tokens, d_model):
            raise ValueError("ring geometry does not match the file")
        self._code = int(self._ctl[5])
        self._dtype = _CODE_DTYPE[self._code]
        self._hdr = self._ctl[:_HDR]
        self._slots = self._ctl[_HDR:].reshape(num_chunks, _SLOT_WORDS)
        self._data = np.memmap(str(dat), dtype=_CODE_NP[self._code], mode="r+",
                               shape=(num_chunks, chunk_size_tokens, d_model))
        self._lock_fd = open(str(lock), "rb")
        self._backoff_n = 0
        self._registered = False

    # ------------------------------------------------------------------ properties
    @property
    def dtype(self) -> torch.dtype:
        return self._dtype

    @property
    def num_chunks(self) -> int:
        return self._n

    @property
    def chunk_size_tokens(self) -> int:
        return self._T

    @property
    def num_producers(self) -> int:
        return int(self._hdr[6])

    @property
    def done_count(self) -> int:
        return int(self._hdr[7])

    @property
    def target_chunks(self) -> int:
        return int(self._hdr[8])

    @property
    def next_claim_seq(self) -> int:
        return int(self._hdr[9])

    # ------------------------------------------------------------------ producer side
    def allocate_write_chunk(self, stop_check: Callable[[], bool] | None = None) -> tuple[int, int] | None:
        """Claim a FREE slot: (slot, seq_no), or None when the global quota is used up or
        `stop_check()` says to stop while waiting for a free slot."""
        while True:
            with self._locked():
                if int(self._hdr[9]) >= int(self._hdr[8]):
                    return None
                free = np.flatnonzero(self._slots[:, 0] == ChunkState.FREE)
                if free.size:
                    i = int(free[0])
                    seq = int(self._hdr[9])
                    self._hdr[9] = seq + 1
                    self._slots[i, 0] = ChunkState.WRITING
                    self._slots[i, 3] = seq
                    self._ctl.flush()
                    self._backoff_n = 0
                    return i, seq
            if stop_check is not None and stop_check():
                return None
            time.sleep(self._backoff())

    def abort_write_chunk(self, chunk_idx: int) -> None:
        with self._locked():
            if int(self._slots[chunk_idx, 0]) != ChunkState.WRITING:
                raise RuntimeError(f"abort_write_chunk on slot {chunk_idx} in state "
                                   f"{ChunkState(int(self._slots[chunk_idx, 0])).name}")
            self._slots[chunk_idx, 0] = ChunkState.FREE
            self._ctl.flush()

    def write_chunk(self, chunk_idx: int, activations: torch.Tensor, valid_tokens: int, producer_id: int = 0) -> None:
        if int(self._slots[chunk_idx, 0]) != ChunkState.WRITING:
            raise RuntimeError(f"write_chunk on slot {chunk_idx} that is not WRITING")
        rows = min(int(valid_tokens), self._T)
        a = activations[:rows].detach()
        if a.dtype != self._dtype:
            a = a.to(self._dtype)
        if self._registered and a.is_cuda:
            self._slot_tensor(chunk_idx, rows).copy_(a)  # device -> page-locked slot (copy engine)
        else:
            a = a.cpu().contiguous()
            view = a.view(torch.int16).numpy().view(np.uint16) if self._code == 0 else a.numpy()
            self._data[chunk_idx, :rows] = view
        if rows < self._T:
            self._data[chunk_idx, rows:] = 0
        self._slots[chunk_idx, 1] = rows
        self._slots[chunk_idx, 2] = producer_id
        self._ctl.flush()

    def mark_ready(self, chunk_idx: int) -> None:
        with self._locked():
            if int(self._slots[chunk_idx, 0]) != ChunkState.WRITING:
                raise RuntimeError(f"mark_ready on slot {chunk_idx} that is not WRITING")
            self._slots[chunk_idx, 0] = ChunkState.READY
            self._ctl.flush()

    def signal_done(self) -> None:
        with self._locked():
            self._hdr[7] = int(self._hdr[7]) + 1
            self._ctl.flush()

    # ------------------------------------------------------------------ consumer side
    def acquire_up_to(self, n: int, random: bool = True) -> tuple[list[int], float]:
        """Claim up to n READY slots; blocks while none is ready and producers are still running;
        raises StopIteration when none is ready and every producer has signalled done.
        Returns (slots, seconds spent waiting)."""
        waited = 0.0
        while True:
            with self._locked():
                ready = [int(i) for i in np.flatnonzero(self._slots[:, 0] == ChunkState.READY)]
                if ready:
                    if random:
                        _random.shuffle(ready)
                    claim = ready[:n]
                    for i in claim:
                        self._slots[i, 0] = ChunkState.CONSUMING
                    self._ctl.flush()
                    self._backoff_n = 0
                    return claim, waited
                if int(self._hdr[7]) >= int(self._hdr[6]):
                    raise StopIteration
            s = self._backoff()
            waited += s
            time.sleep(s)

    def read_chunk(self, chunk_idx: int) -> tuple[torch.Tensor, int]:
        valid = int(self._slots[chunk_idx, 1])
        raw = np.array(self._data[chunk_idx, :valid])
        t = torch.from_numpy(raw.view(np.int16)).view(torch.bfloat16) if self._code == 0 else torch.from_numpy(raw)
        return t, valid

    def read_chunk_into(self, chunk_idx: int, out: torch.Tensor) -> int:
        """Copy a CONSUMING slot's rows straight into `out` (e.g. a pinned staging buffer)."""
        valid = int(self._slots[chunk_idx, 1])
        src = self._data[chunk_idx, :valid]
        dst = out[:valid]
        if self._code == 0:
            np.copyto(dst.view(torch.int16).numpy().view(np.uint16), src)
        else:
            np.copyto(dst.numpy(), src)
        return valid

    def _slot_tensor(self, chunk_idx: int, rows: int) -> torch.Tensor:
        """Zero-copy tensor over the first `rows` rows of a slot (the ring's own memory)."""
        arr = np.asarray(self._data[chunk_idx, :rows])
        return torch.from_numpy(arr.view(np.int16)).view(torch.bfloat16) if self._code == 0 else torch.from_numpy(arr)

    def chunk_view(self, chunk_idx: int) -> tuple[torch.Tensor, int]:
        """Zero-copy tensor of a CONSUMING slot's valid rows, valid only until the slot is
        released (with `register_for_device_copies()` a non-blocking copy to the device reads it
        directly; release the slot only after that copy completed)."""
        valid = int(self._slots[chunk_idx, 1])
        return self._slot_tensor(chunk_idx, valid), valid

    @property
    def registered(self) -> bool:
        return self._registered

    def register_for_device_copies(self) -> bool:
        """Page-lock the data mapping for the CUDA copy engines of every device of this process
        (cudaHostRegister, portable).  Returns False, leaving the pageable path, if it is refused."""
        if self._registered:
            return True
        from saelens_b200 import ops

        if not ops.available():
            return False
        # a refusal (e.g. a mapping of a file on a disk filesystem) keeps the staging-copy path
        self._registered = ops.native().host_register(self._data.ctypes.data, self._data.nbytes) == 0
        return self._registered

    def release_chunk(self, chunk_idx: int) -> None:
        with self._locked():
            if int(self._slots[chunk_idx, 0]) != ChunkState.CONSUMING:
                raise RuntimeError(f"release_chunk on slot {chunk_idx} that is not CONSUMING")
            self._slots[chunk_idx, 0] = ChunkState.FREE
            self._ctl.flush()

    # ------------------------------------------------------------------ monitoring / control
    def queue_counts(self) -> dict[str, int]:
        st = np.asarray(self._slots[:, 0])
        return {s.name.lower(): int((st == s).sum()) for s in ChunkState}

    def snapshot(self) -> dict:
        st = np.asarray(self._slots[:, 0])
        return {"counts": {s.name.lower(): int((st == s).sum()) for s in ChunkState},
                "ready_indices": [int(i) for i in np.flatnonzero(st == ChunkState.READY)]}

    def reset_for_restart(self, new_num_producers: int) -> None:
        """Between worker launches (no worker alive): abandoned WRITING slots become FREE, the
        producer count is set for the new topology and the done count restarts at zero."""
        with self._locked():
            w = self._slots[:, 0] == ChunkState.WRITING
            self._slots[w, 0] = ChunkState.FREE
            self._hdr[6] = new_num_producers
            self._hdr[7] = 0
            self._ctl.flush()

    def close(self) -> None:
        if self._registered:
            from saelens_b200 import ops

            torch.cuda.synchronize()
            ops.native().host_unregister(self._data.ctypes.data)
            self._registered = False
        self._ctl.flush()
        self._data.flush()
        self._lock_fd.close()

    def unlink(self) -> None:
        for p in self.paths:
            try:
                p.unlink()
            except FileNotFoundError:
                pass

    @contextmanager
    def _locked(self) -> Iterator[None]:
        fcntl.flock(self._lock_fd, fcntl.LOCK_EX)
        try:
            yield
        finally:
            fcntl.flock(self._lock_fd, fcntl.LOCK_UN)

    def _backoff(self) -> float:
        self._backoff_n = min(self._backoff_n + 1, 10)
        return self._backoff_n * 1e-3
