"""Split-role data path of the prefix-overlap topologies (local overlap, matched DP).

In these layouts the SAE tensor-parallel group of a replica is a prefix of the replica's ranks
and its first rank is also the replica's LM root.  Only that root runs the language model; it
produces each training batch and broadcasts it to the rest of its SAE TP group, so TP members
never repeat the LM forward.  The reference does the same split at the raw-batch level: the
vLLM root reads the tokens and broadcasts them and the captured activations to the SAE-only ranks
over a Gloo CPU group (sae_lens/training/activations_store.py:617-661, 697-738).  Here the batch
moves device to device with one `torch.distributed` broadcast over the SAE TP group (NCCL over
NVLink on GPUs, Gloo on CPU), preceded by a one-element header carrying the row count, where
0 means the data ended.  Every member sees the same batches in the same order.
"""

from __future__ import annotations

from collections.abc import Iterator
from typing import Any

import torch
import torch.distributed as dist


class ReplicaBroadcastProvider:
    def __init__(self, source: Iterator[torch.Tensor] | None, group: dist.ProcessGroup, src: int, d_in: int,
                 dtype: torch.dtype, device: torch.device | str):
        """`source` is the LM root's data provider (None on the other ranks); `src` is the root's
        global rank; batches are [rows, d_in] of `dtype` on `device`."""
        self.source = source
        self.group = group
        self.src = src
        self.d_in = d_in
        self.dtype = dtype
        self.device = torch.device(device)
        self.is_root = dist.get_rank() == src
        if self.is_root and source is None:
            raise ValueError("the broadcasting rank needs a data source")
        self._done = False

    def __iter__(self) -> ReplicaBroadcastProvider:
        return self

    def __next__(self) -> torch.Tensor:
        if self._done:
            raise StopIteration
        hdr = torch.zeros(1, dtype=torch.int64, device=self.device)
        batch: torch.Tensor | None = None
        if self.is_root:
            assert self.source is not None
            try:
                batch = next(self.source)
            except StopIteration:
                batch = None
            if isinstance(batch, dict):
                raise ValueError("the split-role broadcast carries single-hook batches (multi-hook runs use DDP)")
            if batch is not None:
                batch = batch.to(device=self.device, dtype=self.dtype).contiguous()
                hdr.fill_(batch.shape[0])
        dist.broadcast(hdr, src=self.src, group=self.group)
        n = int(hdr.item())
        if n == 0:
            self._done = True
            raise StopIteration
        if batch is None:
            batch = torch.empty(n, self.d_in, dtype=self.dtype, device=self.device)
        dist.broadcast(batch, src=self.src, group=self.group)
        return batch

    def __getattr__(self, name: str) -> Any:
        # timing hooks of the root's store (the trainer reads them when present)
        if name in ("source", "group", "src", "d_in", "dtype", "device", "is_root", "_done"):
            raise AttributeError(name)
        src = self.__dict__.get("source")
        if src is None:
            raise AttributeError(name)
        return getattr(src, name)
