"""NVTX ranges around collectives and compute phases (sae_lens/profiling.py:10-75).

Collective ranges are emitted only for NCCL-backed groups on a CUDA build, so CPU/gloo runs
pay nothing.  Names keep the reference's `nccl:<site>` convention.
"""

from __future__ import annotations

from collections.abc import Iterator
from contextlib import contextmanager
from typing import Any

import torch


def _nvtx_ok() -> bool:
    return torch.cuda.is_available()


def _is_nccl(group: Any) -> bool:
    try:
        import torch.distributed as dist

        if not dist.is_available() or not dist.is_initialized():
            return False
        return dist.get_backend(group) == "nccl"
    except (RuntimeError, ValueError):  # a group this process is not part of
        return False


@contextmanager
def nccl_nvtx_range(name: str, group: Any = None) -> Iterator[None]:
    if _nvtx_ok() and _is_nccl(group):
        torch.cuda.nvtx.range_push(name)
        try:
            yield
        finally:
            torch.cuda.nvtx.range_pop()
    else:
        yield


@contextmanager
def cuda_nvtx_range(name: str) -> Iterator[None]:
    if _nvtx_ok():
        torch.cuda.nvtx.range_push(name)
        try:
            yield
        finally:
            torch.cuda.nvtx.range_pop()
    else:
        yield
