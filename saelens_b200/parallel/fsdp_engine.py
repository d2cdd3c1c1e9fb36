"""Sharded data-parallel (FSDP-style) TopK / BatchTopK training step on several B200s.

Every rank trains on its own rows (data parallel), but the SAE's latents are sharded: rank r owns
latents [r*n, (r+1)*n) with their fp32 master weights, Adam moments and b_enc, so the optimizer
state per GPU is 1/S of a replica's.  b_dec is replicated (updated identically on every rank from
the averaged gradient).  Reference semantics: `FSDP(FULL_SHARD, use_orig_params=True)` around the
training forward (sae_lens/llm_sae_training_runner.py:449-463, sae_lens/saes/sae.py:928-936):
parameter all-gather before the forward, gradient reduce-scatter in the backward, each rank
steps the optimizer on its shard.

One step on rank r (S ranks, one process per GPU, peer memory over NVLink; no NCCL call inside):

  1. encoder GEMM with the parameter all-gather fused in (`gemm_fsdp_tn_bf16`): the bf16 W_enc
     and W_dec live in full [d_sae, d_in] buffers in every rank's symmetric slab, each rank's own
     shard in place.  Copy warps inside the GEMM push the own W_enc and W_dec tiles to every
     peer and flag them; the tcgen05 producer waits per 256-latent tile, starting the walk at the
     rank's own latents.
  2. row top-k over all d_sae latents (or the BatchTopK selection over this rank's batch), sparse
     decode + MSE + dL/dx_hat against the gathered W_dec (after its flags), CSC pair lists.
  3. latent gradients with the reduce-scatter fused into the gradient kernel's stores: the rows
     of latent j are written straight into slot [r] of its owner's landing area; then a release
     flag per (source, owner).
  4. the owner sums its S slots (rank order, 1/S scale) into the shard's gradient and the
     squared norm; one P2P all-reduce averages [gb_enc | b_dec terms | losses | norm part] and
     one sums the firing counts.
  5. clip + row-fused Adam on the shard, writing the new bf16 rows into the slab in place, then
     a P2P all-reduce of the shard's per-latent vectors (folded bias, ||W_dec||) into full
     replicas for the next GEMM's epilogue.

Buffer reuse needs no extra barrier: a rank writes a peer's landing slot (step t+1) only after its
GEMM of step t+1 consumed that peer's weight tiles, which the peer pushes after its own Adam of
step t, which came after it reduced the slots of step t; a peer overwrites this rank's weight
buffers (step t+1) only after this rank's gradient flag of step t, which follows every read of
them in step t.
"""

from __future__ import annotations

from typing import Any

import torch
import torch.distributed as dist
from torch import nn

from saelens_b200.parallel.symm_heap import SymmetricHeap, slab_bytes_needed
from saelens_b200.parallel.tp_engine import _AllReduceBufs
from saelens_b200.training.engine import EngineStepResult, FusedTopKEngine, update_topk_threshold_ema


def _shard_module(sae: Any, rank: int, world: int) -> int:
    """Replace the module's latent-indexed parameters by this rank's contiguous shard."""
    N = sae.W_dec.shape[0]
    if N % world:
        raise ValueError(f"d_sae {N} is not divisible by {world} ranks")
    n = N // world
    sl = slice(rank * n, (rank + 1) * n)
    with torch.no_grad():
        sae.W_dec = nn.Parameter(sae.W_dec.detach()[sl].clone(), requires_grad=False)
        sae.W_enc = nn.Parameter(sae.W_enc.detach()[:, sl].clone(), requires_grad=False)
        sae.b_enc = nn.Parameter(sae.b_enc.detach()[sl].clone(), requires_grad=False)
    return N


class FSDPTopKEngine(FusedTopKEngine):
    # per-latent vectors replicated after each step: folded bias, ||W_dec||, 1 / ||W_dec|| (a subclass
    # may add more, filled by `_vector_parts`); extra fp32 slots at the end of the averaged small vector
    N_VECS = 3

    def _extra_small(self) -> int:
        return 0

    def __init__(self, sae: Any, lr: float, group: dist.ProcessGroup | None, beta1: float = 0.9,
                 beta2: float = 0.999, eps: float = 1e-8, max_grad_norm: float = 1.0,
                 h_buffer_bytes: int = 8 << 30):
        self.group = group
        self.rank = dist.get_rank(group)
        self.size = dist.get_world_size(group)
        if self.size > 8:
            raise ValueError("peer-memory kernels support at most 8 ranks (one NVSwitch domain)")
        self.N_full = _shard_module(sae, self.rank, self.size)
        super().__init__(sae, lr=lr, beta1=beta1, beta2=beta2, eps=eps, max_grad_norm=max_grad_norm,
                         h_buffer_bytes=h_buffer_bytes)
        nat, dev, S, r = self.native, self.device, self.size, self.rank
        n, D, NF = self.N, self.D, self.N_full
        self.k = min(self.k_request(), NF)
        bf, f32 = torch.bfloat16, torch.float32
        # [gb_enc | bsum | bterm | mse | aux | norm part | subclass extras]
        self._small_n = NF + 2 * D + 3 + self._extra_small()
        sizes = [NF * D * 2, NF * D * 2, (NF // 256) * 4, (NF // 256) * 4, S * n * D * 2, S * n * D * 2, S * 4]
        sizes += _AllReduceBufs.nbytes(nat, self._small_n, 4, S) + _AllReduceBufs.nbytes(nat, NF, 4, S)
        sizes += _AllReduceBufs.nbytes(nat, self.N_VECS * NF, 4, S)
        self.heap = SymmetricHeap(group, slab_bytes_needed(sizes) + 65536, dev)
        h = self.heap
        self.wenc_buf = h.alloc((NF, D), bf)
        self.wdec_buf = h.alloc((NF, D), bf)
        self.wenc_flags = h.alloc(NF // 256, torch.int32)
        self.wdec_flags = h.alloc(NF // 256, torch.int32)
        self.land_dec = h.alloc((S, n, D), bf)
        self.land_enc = h.alloc((S, n, D), bf)
        self.gflags = h.alloc(S, torch.int32)
        self.small = _AllReduceBufs(h, nat, self._small_n, f32)
        self.fire = _AllReduceBufs(h, nat, NF, f32)
        self.vecs = _AllReduceBufs(h, nat, self.N_VECS * NF, f32)
        self.wenc_full = h.local(self.wenc_buf)
        self.wdec_full = h.local(self.wdec_buf)
        self.wdec_flags_local = h.local(self.wdec_flags)
        self.gflags_local = h.local(self.gflags)
        self.land_dec_local = h.local(self.land_dec)
        self.land_enc_local = h.local(self.land_enc)
        # the own bf16 shard lives in place in the gathered buffers; Adam writes it there
        own = slice(r * n, (r + 1) * n)
        self.wenc_full[own].copy_(self.w_enc)
        self.wdec_full[own].copy_(self.w_dec)
        self.w_enc, self.w_dec = self.wenc_full[own], self.wdec_full[own]
        # full-width per-latent state for the step (replicated statistics)
        self.counts_f = torch.zeros(NF, dtype=torch.int32, device=dev)
        self.fire_f = torch.zeros(NF, dtype=torch.int32, device=dev)
        self.cursor_f = torch.zeros(NF, dtype=torch.int32, device=dev)
        self.colptr_f = torch.zeros(NF + 1, dtype=torch.int64, device=dev)
        self.dense_colptr = torch.arange(n + 1, dtype=torch.int64, device=dev)
        self._ticket = torch.zeros(1, dtype=torch.int32, device=dev)
        self._epochs: dict[str, int] = {}
        self._all_mask = (1 << S) - 1
        self.collectives = 0
        self._gather_vectors()

    def k_request(self) -> int:
        cfg = self.sae.cfg
        if self.batch_topk:
            return int(min(1024, max(1, round(4 * float(cfg.k)))))
        return int(cfg.k)

    def _epoch(self, name: str) -> int:
        e = self._epochs.get(name, 0) + 1
        self._epochs[name] = e
        return e

    def _ar(self, x: torch.Tensor, area: _AllReduceBufs, name: str, scale: float) -> torch.Tensor:
        self.native.p2p_allreduce(x, scale, self.heap.bases, self.rank, area.land, area.cnt, area.out_buf.offset,
                                  area.flag, self._epoch(name), self._ticket, self.status.tensor)
        self.launches += 1
        self.collectives += 1
        return area.out

    def _vector_parts(self) -> list[torch.Tensor]:
        return [self.bias_eff, self.scale, self.inv_scale]

    def _gather_vectors(self) -> None:
        """Full replicas of the per-latent epilogue vectors (disjoint shards summed exactly)."""
        NF, n, r = self.N_full, self.N, self.rank
        v = torch.zeros(self.N_VECS * NF, dtype=torch.float32, device=self.device)
        for i, part in enumerate(self._vector_parts()):
            v[i * NF + r * n : i * NF + (r + 1) * n] = part
        out = self._ar(v, self.vecs, "vecs", 1.0)
        self.vec_full = [out[i * NF : (i + 1) * NF] for i in range(self.N_VECS)]
        self.bias_full, self.scale_full, self.inv_scale_full = self.vec_full[:3]

    def refresh(self) -> None:
        super().refresh()
        if hasattr(self, "heap"):
            self._gather_vectors()

    def close(self) -> None:
        self.heap.close()

    def _row_chunk(self, B: int) -> int:
        rows = max(128, (self.h_buffer_bytes // (2 * self.N_full)) // 128 * 128)
        return min((B + 127) // 128 * 128, rows)

    # ------------------------------------------------------------------ the step
    @torch.no_grad()
    def step(self, x: torch.Tensor, lr: float | None = None, dead_mask: torch.Tensor | None = None,
             want_sae_out: bool = False, act_freq: torch.Tensor | None = None,
             since_fired: torch.Tensor | None = None, run_aux: bool = False,
             update: bool = True) -> EngineStepResult:
        nat, dev = self.native, self.device
        S, r, n, D, NF, k = self.size, self.rank, self.N, self.D, self.N_full, self.k
        st, tk, bases = self.status.tensor, self._ticket, self.heap.bases
        B = x.shape[0]
        xb = x if (x.dtype == torch.bfloat16 and x.is_contiguous()) else x.to(torch.bfloat16).contiguous()
        ep = self._epoch("step")
        self._mark("start")

        # 1. parameter all-gather fused encoder GEMM + row top-k over all latents
        R = self._row_chunk(B)
        H = torch.empty(min(R, B), NF, dtype=torch.bfloat16, device=dev)
        cm = torch.empty(min(R, B), NF // 32, dtype=torch.bfloat16, device=dev)
        tm = torch.empty(min(R, B), NF // 256, dtype=torch.bfloat16, device=dev)
        vals = torch.empty(B, k, dtype=torch.float32, device=dev)
        idx = torch.empty(B, k, dtype=torch.int32, device=dev)
        aux_on = run_aux and dead_mask is not None
        k_aux = D // 2
        if aux_on:
            assert dead_mask is not None
            dm = dead_mask.to(torch.bool)
            num_dead = dm.sum().to(torch.int32)
            k_aux_dev = torch.minimum(num_dead, torch.tensor(k_aux, dtype=torch.int32, device=dev)).reshape(1)
            aux_scale = torch.clamp(num_dead.float() / k_aux, max=1.0)
            words = (dm.view(NF // 32, 32).to(torch.int64) << torch.arange(32, device=dev, dtype=torch.int64)).sum(1)
            mask_words = torch.where(words >= 2**31, words - 2**32, words).to(torch.int32).contiguous()
            aux_vals = torch.empty(B, k_aux, dtype=torch.float32, device=dev)
            aux_idx = torch.empty(B, k_aux, dtype=torch.int32, device=dev)
        for r0 in range(0, B, R):
            r1 = min(B, r0 + R)
            h, c, t = H[: r1 - r0], cm[: r1 - r0], tm[: r1 - r0]
            first = r0 == 0
            nat.gemm_fsdp_tn_bf16(xb[r0:r1], self.w_enc, bases, r, self.wenc_buf.offset, self.wenc_flags.offset,
                                  first, ep, self.w_dec if first else None, self.wdec_buf.offset,
                                  self.wdec_flags.offset, self.bias_full, self.scale_full if self.rescale else None,
                                  False, h, c, st, tk, 0, tmax=t)
            self._mark("fsdp_encoder_gemm")
            nat.row_topk(h, c, k, None, None, vals[r0:r1], idx[r0:r1], st, tmax=t)
            self._mark("row_topk")
            self.launches += 2
            if aux_on:
                nat.row_topk(h, c, k_aux, k_aux_dev, mask_words, aux_vals[r0:r1], aux_idx[r0:r1], st)
                self.launches += 1
        del H, cm, tm
        if self.batch_topk:
            sel = nat.batch_topk_select(vals, idx, int(round(self.batch_k * B)), self.batch_truncated)
            self.launches += 5
            update_topk_threshold_ema(self.sae, sel)
            self._mark("batch_topk_select")

        # 2. decode + MSE + dL/dx_hat with the gathered W_dec
        nat.p2p_wait_flags(self.wdec_flags_local, ep, st)
        inv = self.inv_scale_full if self.rescale else None
        sae_out = torch.empty(B, D, dtype=torch.bfloat16, device=dev) if (want_sae_out or aux_on) else None
        dxhat = torch.empty(B, D, dtype=torch.bfloat16, device=dev)
        loss_row = torch.empty(B, dtype=torch.float32, device=dev)
        small = torch.zeros(self._small_n, dtype=torch.float32, device=dev)
        gb_enc, bsum, bterm = small[:NF], small[NF : NF + D], small[NF + D : NF + 2 * D]
        resid = torch.empty(B, D, dtype=torch.bfloat16, device=dev) if aux_on else None
        nat.decode_mse(vals, idx, True, inv, self.wdec_full, self.p_bdec, xb, sae_out, resid, dxhat, None, 2.0 / B,
                       loss_row, bsum)
        self.launches += 2
        daux = None
        if aux_on:
            daux = torch.empty(B, D, dtype=torch.bfloat16, device=dev)
            aux_row = torch.empty(B, dtype=torch.float32, device=dev)
            gcoef = (aux_scale * (2.0 * self.aux_coef / B)).reshape(1).contiguous()
            nat.decode_mse(aux_vals, aux_idx, False, inv, self.wdec_full, None, resid, None, None, daux, gcoef, 1.0,
                           aux_row, None)
            small[NF + 2 * D + 1] = self.aux_coef * aux_scale * aux_row.sum() / B
            self.launches += 1
        small[NF + 2 * D] = loss_row.sum() / B
        self._mark("decode_mse")

        # CSC pair lists over all latents
        self.counts_f.zero_()
        self.fire_f.zero_()
        self.cursor_f.zero_()
        nat.csc_count(vals, idx, aux_vals if aux_on else None, aux_idx if aux_on else None, self.counts_f,
                      self.fire_f)
        torch.cumsum(self.counts_f, 0, out=self.colptr_f[1:])
        pairs = torch.empty(B * k + (B * k_aux if aux_on else 0), dtype=torch.int64, device=dev)
        nat.csc_fill(vals, idx, aux_vals if aux_on else None, aux_idx if aux_on else None, self.colptr_f,
                     self.cursor_f, pairs)
        self._mark("csc_build")

        # 3. latent gradients, rows stored into their owners' landing slots; then publish
        nat.latent_grad(self.colptr_f, pairs, vals, aux_vals if aux_on else None, inv, dxhat, daux, xb,
                        self.p_bdec if self.apply_b_dec else None, self.wdec_full, self.wenc_full, self.g_dec,
                        self.g_enc, gb_enc, bterm if self.apply_b_dec else None, None, None, None, None, idx,
                        aux_idx if aux_on else None, 0, -1, True, rs_bases=bases, rs_rank=r,
                        rs_dec_off=self.land_dec.offset, rs_enc_off=self.land_enc.offset, rs_n=n)
        nat.p2p_signal(bases, r, self.gflags.offset, r, self._all_mask, ep)
        self.launches += 4
        self._mark("latent_grad_reduce_scatter")

        # 4. owner: sum the slots; average the small vector; sum the firing counts
        nat.p2p_wait_flags(self.gflags_local, ep, st)
        part = torch.zeros(1, dtype=torch.float32, device=dev)
        nat.p2p_slot_reduce(self.land_dec_local, 1.0 / S, self.g_dec, part)
        nat.p2p_slot_reduce(self.land_enc_local, 1.0 / S, self.g_enc, part)
        small[NF + 2 * D + 2 : NF + 2 * D + 3] = part * S  # summed (not averaged) by the 1/S all-reduce
        self.launches += 3
        red = self._ar(small, self.small, "small", 1.0 / S)
        fired = self._ar(self.fire_f.to(torch.float32), self.fire, "fire", 1.0)
        self._mark("grad_reduce")
        if act_freq is not None:
            act_freq += fired
        if since_fired is not None:
            since_fired.copy_(torch.where(fired > 0, torch.zeros_like(since_fired), since_fired + 1))
        fire_counts = fired.round().to(torch.int32)
        gb_all = red[:NF]
        sumsq = (red[NF + 2 * D + 2] + gb_all.square().sum()).reshape(1)
        self.sumsq = sumsq
        mse, aux_loss = red[NF + 2 * D], red[NF + 2 * D + 1]

        # 5. clip + Adam on the shard, new bf16 rows in place, per-latent vectors regathered
        if update:
            self.step_count += 1
            cur_lr = self.lr if lr is None else lr
            nat.adam_bdec(red[NF : NF + D], red[NF + D : NF + 2 * D] if self.apply_b_dec else None, self.g_bdec,
                          sumsq, self.clip, self.p_bdec, self.m_bdec, self.v_bdec, cur_lr, self.beta1, self.beta2,
                          self.eps, self.step_count, self.max_grad_norm, True)
            nat.adam_rows(self.p_dec, self.m_dec, self.v_dec, self.p_enc, self.m_enc, self.v_enc, self.w_dec,
                          self.w_enc, self.g_dec, self.g_enc, self.p_benc, self.m_benc, self.v_benc,
                          gb_all[r * n : (r + 1) * n].contiguous(), self.dense_colptr, self.clip,
                          self.p_bdec if self.apply_b_dec else None, self.scale, self.inv_scale, self.bias_eff,
                          cur_lr, self.beta1, self.beta2, self.eps, self.step_count, True)
            self.launches += 2
            self._gather_vectors()
            self._mark("adam")
        self.last_loss = mse + aux_loss
        return EngineStepResult(loss=mse + aux_loss, mse_loss=mse, aux_loss=aux_loss, sae_out=sae_out,
                                topk_vals=vals, topk_idx=idx, fire_counts=fire_counts)

    @torch.no_grad()
    def load_weights(self, W_enc: torch.Tensor, W_dec: torch.Tensor, b_enc: torch.Tensor,
                     b_dec: torch.Tensor) -> None:
        """Full ([d_in, d_sae] / [d_sae, d_in] / [d_sae]) or shard-sized tensors; collective."""
        n, r, dev = self.N, self.rank, self.device
        if W_dec.shape[0] == self.N_full and self.N_full != n:
            sl = slice(r * n, (r + 1) * n)
            W_enc, W_dec, b_enc = W_enc[:, sl], W_dec[sl], b_enc[sl]
        super().load_weights(W_enc.to(dev), W_dec.to(dev), b_enc.to(dev), b_dec.to(dev))

    @torch.no_grad()
    def restore_full_module(self) -> None:
        """Give the module the gathered full parameters again (collective; ends the sharding)."""
        full = self.full_weights()
        for name, t in full.items():
            setattr(self.sae, name, nn.Parameter(t, requires_grad=False))

    def full_weights(self) -> dict[str, torch.Tensor]:
        """Gathered fp32 parameters in the reference layout (collective: every rank calls it)."""
        out = {}
        for name, shard, dim in (("W_dec", self.p_dec, 0), ("W_enc", self.p_enc, 0), ("b_enc", self.p_benc, 0)):
            parts = [torch.empty_like(shard) for _ in range(self.size)]
            dist.all_gather(parts, shard.contiguous(), group=self.group)
            full = torch.cat(parts, dim=dim)
            out[name] = full.T.contiguous() if name == "W_enc" else full
        out["b_dec"] = self.p_bdec.clone()
        return out


__all__ = ["FSDPTopKEngine"]
