"""Autograd-aware tensor-parallel collectives for latent-sharded SAEs (portable path).

Counterparts of `tp_allgather` / `tp_allreduce` (sae_lens/distributed.py:404-461) plus a
`tp_copy` whose backward sums the gradient over the TP group.  `tp_copy` is applied to the SAE
input before the local encoder GEMM, so the gradient that reaches a replicated `b_dec` through
the encoder input is the sum over all latent shards, i.e. exactly the TP=1 gradient.
"""

from __future__ import annotations

from typing import Any

import torch
import torch.distributed as dist

from saelens_b200.parallel.profiling import nccl_nvtx_range


class _AllGatherLastDim(torch.autograd.Function):
    @staticmethod
    def forward(ctx: Any, x: torch.Tensor, group: dist.ProcessGroup) -> torch.Tensor:
        ctx.group = group
        ws = dist.get_world_size(group)
        ctx.rank = dist.get_rank(group)
        ctx.width = x.shape[-1]
        parts = [torch.empty_like(x) for _ in range(ws)]
        with nccl_nvtx_range("nccl:tp_allgather", group):
            dist.all_gather(parts, x.contiguous(), group=group)
        return torch.cat(parts, dim=-1)

    @staticmethod
    def backward(ctx: Any, g: torch.Tensor) -> tuple[torch.Tensor, None]:
        s = ctx.rank * ctx.width
        return g[..., s : s + ctx.width].contiguous(), None


class _AllReduceSum(torch.autograd.Function):
    @staticmethod
    def forward(ctx: Any, x: torch.Tensor, group: dist.ProcessGroup) -> torch.Tensor:
        y = x.clone()
        with nccl_nvtx_range("nccl:tp_allreduce", group):
            dist.all_reduce(y, group=group)
        return y

    @staticmethod
    def backward(ctx: Any, g: torch.Tensor) -> tuple[torch.Tensor, None]:
        return g, None


class _CopyToTP(torch.autograd.Function):
    @staticmethod
    def forward(ctx: Any, x: torch.Tensor, group: dist.ProcessGroup) -> torch.Tensor:
        ctx.group = group
        return x

    @staticmethod
    def backward(ctx: Any, g: torch.Tensor) -> tuple[torch.Tensor, None]:
        g = g.contiguous().clone()
        with nccl_nvtx_range("nccl:tp_input_grad_allreduce", ctx.group):
            dist.all_reduce(g, group=ctx.group)
        return g, None


def tp_allgather(x: torch.Tensor, group: dist.ProcessGroup | None) -> torch.Tensor:
    return x if group is None else _AllGatherLastDim.apply(x, group)


def tp_allreduce(x: torch.Tensor, group: dist.ProcessGroup | None) -> torch.Tensor:
    return x if group is None else _AllReduceSum.apply(x, group)


def tp_copy(x: torch.Tensor, group: dist.ProcessGroup | None) -> torch.Tensor:
    return x if group is None else _CopyToTP.apply(x, group)
