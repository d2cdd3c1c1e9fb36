"""Trainer-side data provider over the shared activation ring
(behaviour of sae_lens/training/streaming_activation_provider.py).

The SAE-TP root claims up to `prefetch_chunks` READY slots, copies them to the device, releases
the slots and broadcasts the rows to its TP followers
(`[n_rows]` first, 0 meaning end of stream); every rank shuffles, keeps the remainder of the
previous refill and serves `train_batch_size_tokens` rows per step.  When the ring is page-locked
(`SharedActivationBuffer.register_for_device_copies`) the copy engine reads the slots directly, on
a side stream that runs beside the previous step's kernels; otherwise the rows go through one
pinned staging buffer.  Multi-hook streams store
`num_hooks` interleaved batches and are served as `{hook_name: rows}` dicts.
"""

from __future__ import annotations

import json
import time
from collections.abc import Iterator
from pathlib import Path

import torch
import torch.distributed as dist

from saelens_b200.training.shared_activation_buffer import SharedActivationBuffer


class StreamingActivationProvider:
    def __init__(self, buffer: SharedActivationBuffer, train_batch_size_tokens: int, prefetch_chunks: int,
                 device: torch.device | str, sae_tp_group: dist.ProcessGroup | None = None, sae_tp_rank: int = 0,
                 sae_tp_root_global_rank: int = 0, d_model: int = 0, dtype: torch.dtype = torch.float32,
                 shm_log_path: Path | None = None, shuffle: bool = True, random_chunks: bool = True,
                 buffer_monitor_path: Path | None = None, hook_names: list[str] | None = None,
                 generator: torch.Generator | None = None) -> None:
        self._buffer = buffer
        self._batch = train_batch_size_tokens
        self._prefetch = prefetch_chunks
        self._device = torch.device(device)
        self._dtype = dtype
        self._group = sae_tp_group
        self._tp_rank = sae_tp_rank
        self._root = sae_tp_root_global_rank
        self._d_model = d_model
        self._shuffle = shuffle
        self._random_chunks = random_chunks
        self._hooks = hook_names
        self._n_hooks = len(hook_names) if hook_names else 1
        self._gen = generator
        self._pool: torch.Tensor | None = None
        self._start = 0
        self._consumed = 0
        self._wait_s = 0.0
        self._transfer_s = 0.0
        self._t0 = time.time()
        self._staging: torch.Tensor | None = None
        self._direct = bool(getattr(buffer, "registered", False)) and self._device.type == "cuda" and sae_tp_rank == 0
        self._copy_stream = torch.cuda.Stream(self._device) if self._direct else None
        self._staging_free: torch.cuda.Event | None = None  # set after the last H2D from staging
        self._log_path = shm_log_path if sae_tp_rank == 0 else None
        self._mon_path = buffer_monitor_path if sae_tp_rank == 0 else None
        self._mon_step = 0
        for p in (self._log_path, self._mon_path):
            if p is not None:
                p.parent.mkdir(parents=True, exist_ok=True)
                p.write_text("")

    def __iter__(self) -> Iterator[torch.Tensor | dict[str, torch.Tensor]]:
        return self

    @property
    def consumed_tokens(self) -> int:
        return self._consumed

    def _avail(self) -> int:
        return 0 if self._pool is None else self._pool.shape[0] - self._start

    def __next__(self) -> torch.Tensor | dict[str, torch.Tensor]:
        need = self._batch * self._n_hooks
        if self._avail() >= need:
            return self._take()
        try:
            self._refill()
        except StopIteration:
            if self._avail() > 0:
                return self._take()
            raise
        if self._avail() == 0:
            raise StopIteration
        return self._take()

    def consume_last_data_timing(self) -> dict[str, float]:
        out = {"vllm_step_time_s": self._wait_s, "transfer_time_s": self._transfer_s}
        self._wait_s = self._transfer_s = 0.0
        return out

    def _log(self, path: Path | None, rec: dict) -> None:
        if path is None:
            return
        rec["elapsed_s"] = time.time() - self._t0
        with open(path, "a") as f:
            f.write(json.dumps(rec) + "\n")

    def _bcast_count(self, n: int) -> int:
        t = torch.tensor([n], dtype=torch.int64, device=self._device)
        dist.broadcast(t, src=self._root, group=self._group)
        return int(t.item())

    def _refill(self) -> None:
        if self._tp_rank == 0:
            if self._mon_path is not None:
                self._mon_step += 1
                snap = self._buffer.snapshot()
                self._log(self._mon_path, {"refill_step": self._mon_step, "ready_count": snap["counts"]["ready"],
                                           "ready_indices": snap["ready_indices"], "counts": snap["counts"]})
            t0 = time.perf_counter()
            try:
                idx, waited = self._buffer.acquire_up_to(self._prefetch, random=self._random_chunks)
            except StopIteration:
                self._log(self._log_path, {"event": "refill_exhausted", "wait_time_s": time.perf_counter() - t0})
                if self._group is not None:
                    self._bcast_count(0)
                raise
            t1 = time.perf_counter()
            rows_max = len(idx) * self._buffer.chunk_size_tokens
            D = self._d_model or self._buffer._D
            if self._direct:
                new = self._copy_direct(idx, D)
            else:
                new = self._copy_staged(idx, D, rows_max)
            n = new.shape[0]
            if self._group is not None:
                self._bcast_count(n)
                dist.broadcast(new, src=self._root, group=self._group)
            self._wait_s, self._transfer_s = waited, time.perf_counter() - t1
            self._log(self._log_path, {"event": "refill_complete", "chunks": idx, "new_tokens": n,
                                       "wait_time_s": waited, "transfer_time_s": self._transfer_s})
        else:
            t0 = time.perf_counter()
            n = self._bcast_count(0)
            if n == 0:
                raise StopIteration
            new = torch.empty(n, self._d_model, dtype=self._dtype, device=self._device)
            dist.broadcast(new, src=self._root, group=self._group)
            self._wait_s, self._transfer_s = 0.0, time.perf_counter() - t0
        if self._n_hooks > 1:
            new = self._regroup_hooks(new)
        elif self._shuffle:
            perm = torch.randperm(new.shape[0], device=self._device, generator=self._gen)
            if new.is_cuda:
                # the leftover pool rows followed by the shuffled new rows, gathered in one pass
                from saelens_b200 import ops

                rest = self._pool[self._start :] if self._avail() > 0 else None
                r = 0 if rest is None else rest.shape[0]
                idx = perm + r if r == 0 else torch.cat([torch.arange(r, device=new.device), perm + r])
                self._pool = ops.gather_rows(rest, new, idx) if rest is not None else ops.gather_rows(new, None, idx)
                self._start = 0
                return
            new = new[perm]
        if self._avail() > 0:
            assert self._pool is not None
            new = torch.cat([self._pool[self._start :], new])
        self._pool, self._start = new, 0

    def _copy_direct(self, idx: list[int], D: int) -> torch.Tensor:
        """Claimed page-locked slots -> device on the copy stream; the slots are released once the
        copies completed, and the compute stream waits for them before it reads the rows."""
        assert self._copy_stream is not None
        views = [self._buffer.chunk_view(i) for i in idx]
        n = sum(v for _, v in views)
        cur = torch.cuda.current_stream(self._device)
        with torch.cuda.stream(self._copy_stream):
            raw = torch.empty(n, D, dtype=self._buffer.dtype, device=self._device)
            o = 0
            for t, v in views:
                raw[o : o + v].copy_(t, non_blocking=True)
                o += v
            done = torch.cuda.Event()
            done.record(self._copy_stream)
        done.synchronize()  # the slots have been read
        for i in idx:
            self._buffer.release_chunk(i)
        cur.wait_event(done)
        raw.record_stream(cur)
        return raw.to(self._dtype)

    def _copy_staged(self, idx: list[int], D: int, rows_max: int) -> torch.Tensor:
        """Claimed slots -> one pinned staging buffer (host copy) -> device; the slots are free as
        soon as the host copy is done."""
        if self._staging_free is not None:
            self._staging_free.synchronize()  # the previous async copy out of staging is done
        if self._staging is None or self._staging.shape[0] < rows_max:
            self._staging = torch.empty(rows_max, D, dtype=self._buffer.dtype,
                                        pin_memory=self._device.type == "cuda")
        n = 0
        for i in idx:
            n += self._buffer.read_chunk_into(i, self._staging[n:])
            self._buffer.release_chunk(i)
        if self._device.type == "cuda":
            new = self._staging[:n].to(self._device, non_blocking=True).to(self._dtype)
            self._staging_free = torch.cuda.Event()
            self._staging_free.record()
        else:
            new = self._staging[:n].to(self._dtype, copy=True)
        return new

    def _regroup_hooks(self, new: torch.Tensor) -> torch.Tensor:
        """Rows arrive as [hook0 block, hook1 block, ...] per producer step of `batch` tokens;
        shuffle the token order identically for every hook and keep the block interleave."""
        H, b = self._n_hooks, self._batch
        steps = new.shape[0] // (H * b)
        if steps == 0:
            return new
        blocks = new[: steps * H * b].view(steps, H, b, -1)
        if self._shuffle:
            perm = torch.randperm(steps * b, device=new.device, generator=self._gen)
            per_hook = blocks.permute(1, 0, 2, 3).reshape(H, steps * b, -1)[:, perm]
            blocks = per_hook.view(H, steps, b, -1).permute(1, 0, 2, 3)
        return torch.cat([blocks.reshape(-1, new.shape[-1]), new[steps * H * b :]])

    def _take(self) -> torch.Tensor | dict[str, torch.Tensor]:
        assert self._pool is not None
        need = self._batch * self._n_hooks
        take = min(need, self._avail())
        out = self._pool[self._start : self._start + take]
        self._start += take
        self._consumed += take // self._n_hooks
        if self._n_hooks > 1 and self._hooks is not None:
            per = take // self._n_hooks
            return {h: out[i * per : (i + 1) * per] for i, h in enumerate(self._hooks)}
        return out
