"""CPU reference implementations of the peer-memory collective algorithms, over any
torch.distributed backend (tests run them on gloo ranks).  Each follows the data movement of its
CUDA kernel, so the host-side arithmetic (ownership, offsets, ordering, tie rules, scaling) is
testable without GPUs:

* `two_shot_allreduce`   - ops/csrc/p2p.cu allreduce_kernel: chunk c is owned by rank c % S; owners
                           sum the S contributions in rank order, scale, round to the element type
                           and return the chunk (with its sum of squares) to every rank.
* `decode_reduce_scatter`- ops/csrc/sparse.cu decode_rs_kernel: row b belongs to rank b // Bo; the
                           owner sums the fp32 partial rows in rank order, adds b_dec, and forms
                           the loss rows and dL/dx_hat, which every rank receives.
* `candidate_merge`      - ops/csrc/topk.cu topk_exchange_merge_kernel: global per-row top-k over
                           every rank's candidates, ties broken by the smaller global latent id;
                           returns this rank's keep mask.
* `route_rows`           - ops/csrc/p2p.cu route_rows_kernel: producer rows to consumers by the
                           shard-routing table, normalised and cast to bf16, assembled in producer
                           order.
* `fsdp_reduce_scatter`  - the gradient reduce-scatter of parallel/fsdp_engine.py (ops/csrc/sparse.cu
                           latent_rows_kernel stores + ops/csrc/p2p.cu slot_reduce_kernel): rank r
                           stores the bf16 row of latent j in slot [r][j - o*n] of owner o = j // n;
                           the owner sums its S slots in rank order, times 1/S, rounded to bf16.
* `sharded_batch_topk`   - the latent-sharded BatchTopK of parallel/tp_engine.py (ops/csrc/topk.cu
                           batch_* kernels): per-shard row candidates, summed 16-bit key histogram,
                           threshold, summed [S, B] tie counts, ties kept in (row, global latent)
                           order.
"""

from __future__ import annotations


import torch
import torch.distributed as dist

from saelens_b200.parallel.shard_routing import compute_routing_table


def _gather_all(t: torch.Tensor, group: dist.ProcessGroup | None) -> list[torch.Tensor]:
    out = [torch.empty_like(t) for _ in range(dist.get_world_size(group))]
    dist.all_gather(out, t.contiguous(), group=group)
    return out


def two_shot_allreduce(x: torch.Tensor, group: dist.ProcessGroup | None = None, chunk: int = 4096,
                       scale: float = 1.0) -> tuple[torch.Tensor, torch.Tensor]:
    """Returns (result in x.dtype, per-chunk sum of squares of the rounded result)."""
    S, r = dist.get_world_size(group), dist.get_rank(group)
    n = x.numel()
    nch = (n + chunk - 1) // chunk
    flat = x.reshape(-1)
    # phase A: every chunk goes to its owner (an all-gather moves the same bytes on CPU ranks)
    parts = _gather_all(flat, group)
    out = torch.empty_like(flat)
    sq = torch.zeros(nch, dtype=torch.float32)
    mine = torch.zeros_like(flat)
    owned = torch.zeros(n, dtype=torch.bool)
    for c in range(r, nch, S):
        lo, hi = c * chunk, min(n, (c + 1) * chunk)
        acc = torch.zeros(hi - lo, dtype=torch.float32)
        for s in range(S):
            acc += parts[s][lo:hi].float()
        v = (acc * scale).to(x.dtype)
        mine[lo:hi] = v
        owned[lo:hi] = True
        sq[c] = v.float().square().sum()
    # phase B: owners hand their chunks to everyone
    got = _gather_all(torch.where(owned, mine, torch.zeros_like(mine)), group)
    sq_all = _gather_all(sq, group)
    for c in range(nch):
        o = c % S
        lo, hi = c * chunk, min(n, (c + 1) * chunk)
        out[lo:hi] = got[o][lo:hi]
        sq[c] = sq_all[o][c]
    return out.reshape(x.shape), sq


def decode_reduce_scatter(partial: torch.Tensor, b_dec: torch.Tensor | None, target_own: torch.Tensor,
                          grad_coef: float, group: dist.ProcessGroup | None = None
                          ) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """partial [B, D] fp32 (this rank's partial reconstruction of every row); target_own [Bo, D].
    Returns (sae_out of owned rows, loss per owned row, dL/dx_hat of all B rows in bf16)."""
    S, r = dist.get_world_size(group), dist.get_rank(group)
    B, D = partial.shape
    Bo = B // S
    parts = _gather_all(partial, group)
    acc = torch.zeros(Bo, D, dtype=torch.float32)
    for s in range(S):  # rank order, as the owner reduces its landing area
        acc += parts[s][r * Bo : (r + 1) * Bo]
    xh = acc + (b_dec.float() if b_dec is not None else 0.0)
    err = xh - target_own.float()
    loss_row = err.square().sum(-1)
    dx_own = (err * grad_coef).to(torch.bfloat16)
    dx = torch.cat(_gather_all(dx_own, group))
    return xh, loss_row, dx


def candidate_merge(vals: torch.Tensor, idx: torch.Tensor, n_local: int, k: int,
                    group: dist.ProcessGroup | None = None) -> torch.Tensor:
    """vals/idx [B, k] this rank's candidates (local ids, -1 = none).  Keep mask of this rank's
    entries in the global per-row top-k (ties at the k-th value: smaller global id first)."""
    S, r = dist.get_world_size(group), dist.get_rank(group)
    all_v, all_i = _gather_all(vals, group), _gather_all(idx, group)
    B = vals.shape[0]
    keep = torch.zeros_like(idx, dtype=torch.bool)
    for b in range(B):
        entries = []
        for s in range(S):
            for i in range(all_i[s].shape[1]):
                li = int(all_i[s][b, i])
                if li >= 0:
                    entries.append((-float(all_v[s][b, i]), s * n_local + li, s, i))
        entries.sort()
        for _, _, s, i in entries[:k]:
            if s == r:
                keep[b, i] = True
    return keep


def route_rows(x: torch.Tensor | None, producers: list[int], consumers: list[int], batch_rows: int,
               normalize: str = "none", scale: float = 1.0, group: dist.ProcessGroup | None = None
               ) -> torch.Tensor | None:
    """Producers pass their [batch_rows, d] rows; consumers get their assembled bf16 rows."""
    rank = dist.get_rank(group)
    P, Q = len(producers), len(consumers)
    routes = compute_routing_table(P, Q, batch_rows)
    d = x.shape[1] if x is not None else None
    dims = _gather_all(torch.tensor([d if d is not None else -1]), group)
    d = max(int(t) for t in dims)
    send = torch.zeros(batch_rows, d) if x is None else x.float()
    if x is not None and normalize == "unit_norm":
        send = send / send.norm(dim=-1, keepdim=True).clamp(min=1e-12) * scale
    elif x is not None and normalize == "scale":
        send = send * scale
    allx = _gather_all(send.to(torch.bfloat16), group)
    if rank not in consumers:
        return None
    c = consumers.index(rank)
    parts = [allx[producers[rt.producer_idx]][rt.row_start : rt.row_end]
             for rt in sorted((rt for rt in routes if rt.consumer_idx == c), key=lambda rt: rt.producer_idx)]
    return torch.cat(parts)


def fsdp_reduce_scatter(grad_rows: torch.Tensor, group: dist.ProcessGroup | None = None) -> torch.Tensor:
    """grad_rows [N, D]: this rank's gradient rows of every latent.  Returns this rank's shard
    [N / S, D] of the rank-mean, with the kernels' rounding (bf16 parts, fp32 sum, bf16 result)."""
    S, r = dist.get_world_size(group), dist.get_rank(group)
    N, D = grad_rows.shape
    n = N // S
    mine = grad_rows.to(torch.bfloat16)
    # slots[o][src] on the owner: every rank's rows of owner o's latents (an all-gather moves the
    # same bytes on CPU ranks as the P2P stores into the owners' landing areas)
    every = _gather_all(mine, group)
    acc = torch.zeros(n, D, dtype=torch.float32)
    for src in range(S):  # rank order, as the owner's slot reduce
        acc += every[src][r * n : (r + 1) * n].float()
    return (acc * (1.0 / S)).to(torch.bfloat16)


def bf16_keys(v: torch.Tensor) -> torch.Tensor:
    """Order-preserving 16-bit keys of bf16 values (int64): positive values map above 0x8000."""
    b = v.to(torch.bfloat16).view(torch.int16).to(torch.int64) & 0xFFFF
    return torch.where(b >= 0x8000, (~b) & 0xFFFF, b | 0x8000)


def sharded_batch_topk(h_local: torch.Tensor, k_batch: float, k_cap: int,
                       group: dist.ProcessGroup | None = None) -> torch.Tensor:
    """h_local [B, n_local]: this shard's pre-activations (bf16-exact).  Returns the bool mask of
    this shard's entries among the round(k_batch * B) largest positive values of the whole
    [B, S * n_local] batch (only the per-shard per-row top-k_cap are candidates)."""
    S, r = dist.get_world_size(group), dist.get_rank(group)
    B, n = h_local.shape
    K = int(round(k_batch * B))
    cv, ci = h_local.float().topk(min(k_cap, n), dim=1)
    keys = bf16_keys(cv)
    pos = cv > 0
    hist = torch.bincount(keys[pos], minlength=65536).to(torch.int64)
    dist.all_reduce(hist, group=group)
    above_cum = hist.flip(0).cumsum(0).flip(0)  # count of keys >= key
    hit = (above_cum >= K).nonzero()
    if K > 0 and len(hit) > 0 and int(hit.max()) > 0x8000:
        key = int(hit.max())
        budget = K - int(above_cum[key + 1]) if key < 65535 else K
    else:
        key, budget = 0x8000, 0
    tie = pos & (keys == key)
    ties = torch.zeros(S, B, dtype=torch.int64)
    ties[r] = tie.sum(1)
    dist.all_reduce(ties, group=group)
    row_tot = ties.sum(0)
    prefix = row_tot.cumsum(0) - row_tot + ties[:r].sum(0)
    mask = torch.zeros(B, n, dtype=torch.bool)
    for b in range(B):
        order = ci[b].argsort()  # ties ranked by local index inside the row
        seen = 0
        for j in order.tolist():
            if not pos[b, j]:
                continue
            if keys[b, j] > key:
                mask[b, ci[b, j]] = True
            elif keys[b, j] == key:
                if prefix[b] + seen < budget:
                    mask[b, ci[b, j]] = True
                seen += 1
    return mask


__all__ = ["two_shot_allreduce", "decode_reduce_scatter", "candidate_merge", "route_rows", "bf16_keys",
           "sharded_batch_topk", "fsdp_reduce_scatter"]
