"""Megatron-style tensor parallelism for the producer LM (the role vLLM's tensor parallelism plays
in the reference's producer: sae_lens/vllm_model.py:669-741, with the sharded hooks gathered as in
sae_lens/training/activations_store.py:917-944).

`shard_lm_tensor_parallel(model, group)` keeps on rank r of T:
* attention: query heads [r H/T, (r+1) H/T) and K/V heads [r KV/T, (r+1) KV/T) (rows of the q / k /
  v projections) and the matching input columns of the output projection;
* MLP: rows [r d_mlp/T, (r+1) d_mlp/T) of the gate / up projections and the matching input
  columns of the down projection;
* embeddings, norms and the unembedding replicated.
After the output and down projections the ranks' partial sums are all-reduced over the group and
the bias is added once, after the sum, so every residual-stream hook (`hook_resid_*`,
`hook_attn_out`, `hook_mlp_out`) holds the full activation on every rank.  The head- or
column-sharded hooks (`attn.hook_q/k/v/z`, `attn.hook_rot_q/k`, `mlp.hook_pre/post`) are gathered
only when a hook is attached: the shards are all-gathered, the hook runs on the full tensor, and
the rank keeps its shard of the (possibly edited) result.  Every rank of the group must run the
same forward with the same hooks (the collectives are issued in the same order).
"""

from __future__ import annotations

from typing import Any

import torch
import torch.distributed as dist
from torch import nn


class TPContext:
    def __init__(self, group: dist.ProcessGroup):
        self.group = group
        self.rank = dist.get_rank(group)
        self.size = dist.get_world_size(group)
        self.all_reduces = 0
        self.gathers = 0

    def all_reduce(self, y: torch.Tensor) -> torch.Tensor:
        y = y.contiguous()
        dist.all_reduce(y, group=self.group)
        self.all_reduces += 1
        return y

    def gather(self, t: torch.Tensor, dim: int) -> torch.Tensor:
        t = t.contiguous()
        parts = [torch.empty_like(t) for _ in range(self.size)]
        dist.all_gather(parts, t, group=self.group)
        self.gathers += 1
        return torch.cat(parts, dim=dim)

    def hooked(self, hp: nn.Module, t: torch.Tensor, dim: int) -> torch.Tensor:
        full = hp(self.gather(t, dim))
        w = t.shape[dim]
        return full.narrow(dim, self.rank * w, w).contiguous()


def _rows(p: torch.Tensor, lo: int, hi: int) -> nn.Parameter:
    return nn.Parameter(p.detach()[lo:hi].clone(), requires_grad=p.requires_grad)


def _cols(p: torch.Tensor, lo: int, hi: int) -> nn.Parameter:
    return nn.Parameter(p.detach()[:, lo:hi].contiguous().clone(), requires_grad=p.requires_grad)


@torch.no_grad()
def shard_lm_tensor_parallel(model: Any, group: dist.ProcessGroup, sync_from_root: bool = True) -> Any:
    """Shard `model` (a HookedLM) in place for tensor parallelism over `group`; returns the model.
    With `sync_from_root` the group's first rank's weights are broadcast first, so members that
    initialised the model independently (random init) still shard one model."""
    ctx = TPContext(group)
    if sync_from_root:
        root = dist.get_global_rank(group, 0)
        for t in list(model.parameters()) + list(model.buffers()):
            dist.broadcast(t.data, src=root, group=group)
    T, r = ctx.size, ctx.rank
    cfg = model.cfg
    H, KV, dh, dm = cfg.n_heads, cfg.n_key_value_heads, cfg.d_head, cfg.d_mlp
    if H % T or KV % T or dm % T:
        raise ValueError(f"tensor parallelism over {T} ranks needs n_heads ({H}), n_key_value_heads ({KV}) "
                         f"and d_mlp ({dm}) divisible by {T}")
    hl, kvl, ml = H // T, KV // T, dm // T
    for blk in model.blocks:
        at = blk.attn
        at.q.weight = _rows(at.q.weight, r * hl * dh, (r + 1) * hl * dh)
        at.k.weight = _rows(at.k.weight, r * kvl * dh, (r + 1) * kvl * dh)
        at.v.weight = _rows(at.v.weight, r * kvl * dh, (r + 1) * kvl * dh)
        for lin, lo, hi in ((at.q, r * hl * dh, (r + 1) * hl * dh), (at.k, r * kvl * dh, (r + 1) * kvl * dh),
                            (at.v, r * kvl * dh, (r + 1) * kvl * dh)):
            if lin.bias is not None:
                lin.bias = _rows(lin.bias, lo, hi)
                lin._bias_f32 = None
        at.o.weight = _cols(at.o.weight, r * hl * dh, (r + 1) * hl * dh)
        if at.o.bias is not None:
            at.o_bias_after = at.o.bias.detach().clone()
            at.o.bias = None
            at.o._bias_f32 = None
        at.n_heads_local, at.n_kv_local, at.tp = hl, kvl, ctx
        mlp = blk.mlp
        if mlp.gated:
            mlp.gate.weight = _rows(mlp.gate.weight, r * ml, (r + 1) * ml)
            if mlp.gate.bias is not None:
                mlp.gate.bias = _rows(mlp.gate.bias, r * ml, (r + 1) * ml)
                mlp.gate._bias_f32 = None
        mlp.up.weight = _rows(mlp.up.weight, r * ml, (r + 1) * ml)
        if mlp.up.bias is not None:
            mlp.up.bias = _rows(mlp.up.bias, r * ml, (r + 1) * ml)
            mlp.up._bias_f32 = None
        mlp.down.weight = _cols(mlp.down.weight, r * ml, (r + 1) * ml)
        if mlp.down.bias is not None:
            mlp.down_bias_after = mlp.down.bias.detach().clone()
            mlp.down.bias = None
            mlp.down._bias_f32 = None
        mlp.d_mlp_local, mlp.tp = ml, ctx
        for lin in (at.q, at.k, at.v, at.o, mlp.up, mlp.down) + ((mlp.gate,) if mlp.gated else ()):
            lin._native_ok = lin.weight.shape[1] % 8 == 0  # the GEMM's K is the (sliced) input width
    model.tp = ctx
    return model


__all__ = ["TPContext", "shard_lm_tensor_parallel"]
