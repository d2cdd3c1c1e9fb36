"""Host-to-device prefetch for any data provider (an iterator of activation batches).

`DevicePrefetcher(provider, device)` yields the provider's batches already on `device`.  The copy
of batch i+1 (from pinned host memory, `non_blocking=True`) is issued on a dedicated copy stream
while the caller's stream still works on batch i, so the transfer overlaps the training step
instead of preceding it.  The caller's stream waits on the copy's event before it touches the
batch, and the device tensor is tied to that stream for the caching allocator.  The reference
copies each batch on the compute stream (`next(self.data_provider).to(device)`,
sae_lens/training/sae_trainer.py:281); the streaming provider there stages one chunk at a time
(sae_lens/training/streaming_activation_provider.py:164-261).
"""

from __future__ import annotations

from collections import deque
from collections.abc import Iterator
from typing import Any

import torch


class DevicePrefetcher:
    def __init__(self, provider: Iterator[Any], device: torch.device | str, depth: int = 1,
                 dtype: torch.dtype | None = None):
        self.provider = provider
        self.device = torch.device(device)
        self.depth = max(1, int(depth))
        self.dtype = dtype
        self.cuda = self.device.type == "cuda"
        self.stream = torch.cuda.Stream(device=self.device) if self.cuda else None
        self._q: deque[tuple[Any, Any, Any]] = deque()
        self._done = False

    def __iter__(self) -> DevicePrefetcher:
        return self

    def _issue(self) -> None:
        if self._done:
            return
        try:
            host = next(self.provider)
        except StopIteration:
            self._done = True
            return
        if not self.cuda:
            self._q.append((host.to(self.device, dtype=self.dtype or host.dtype), None, host))
            return
        assert self.stream is not None
        # the copy may only start once the caller's stream has finished with what came before
        self.stream.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(self.stream):
            dev = host.to(self.device, non_blocking=True)
            if self.dtype is not None and dev.dtype != self.dtype:
                dev = dev.to(self.dtype)
            ev = torch.cuda.Event()
            ev.record(self.stream)
        self._q.append((dev, ev, host))  # the host buffer stays referenced until the copy is consumed

    def __next__(self) -> torch.Tensor:
        while len(self._q) < self.depth + 1 and not self._done:
            self._issue()
        if not self._q:
            raise StopIteration
        dev, ev, _host = self._q.popleft()
        if ev is not None:
            cur = torch.cuda.current_stream(self.device)
            cur.wait_event(ev)
            dev.record_stream(cur)
        return dev

    def __getattr__(self, name: str) -> Any:
        # timing hooks and other attributes of the wrapped provider stay reachable
        if name in ("provider", "device", "depth", "dtype", "cuda", "stream", "_q", "_done"):
            raise AttributeError(name)
        return getattr(self.provider, name)
