"""Latent-sharded tensor-parallel TopK training step on several B200s.

Each of the S ranks owns d_sae/S latents (W_enc^T / W_dec rows, b_enc) plus a replica of b_dec,
and receives B/S rows of the batch (row-sharded input; `input_layout="replicated"` accepts the
full batch on every rank instead, as the reference's TP path does).  One step
(reference semantics: sae_lens/saes/topk_sae.py:615-674 with sae_lens/distributed.py:404-461):

  1. all-gather the input rows                       X [B, d_in]
  2. local encoder GEMM + per-row top-k of the shard  (k candidates per row and rank)
  3. all-gather the candidates (S*k per row instead of the reference's B x d_sae all-gather of
     pre-activations), exact global top-k per row; each rank keeps its own winners
  4. local sparse decode -> reduce-scatter of the fp32 partial reconstructions to row owners,
     then b_dec add + MSE + dL/dx_hat on owned rows
  5. all-gather dL/dx_hat, local latent gradients (CSC)
  6. one all-reduce of [sum_b dL/dx_hat, sum_j gb_enc W_enc, grad sq-norm, loss] (2*d_in+3
     floats), then b_dec gradient, clip and Adam exactly as on one GPU

Two implementations of the exchanges share the compute kernels:

* `fused=True` (default on CUDA): every exchange is a peer-memory kernel over NVLink with the
  compute it serves: the input all-gather runs inside the tcgen05 encoder GEMM (copy warps push
  the own rows, the TMA producer waits per m-tile), the candidate all-gather inside the merge,
  the reduce-scatter of partial reconstructions inside the decode (with b_dec, MSE and the
  dL/dx_hat broadcast), and the statistics all-reduce is a two-shot P2P kernel.  No NCCL call
  runs inside a step.
* `fused=False`: the same step with NCCL collectives between the kernels (the baseline).

BatchTopK (keep the k*B largest activations of the TP batch, sae_lens/saes/batchtopk_sae.py:13-33;
the reference's TP path all-gathers the [B, d_sae] pre-activations and selects on every rank)
replaces step 3: each shard lists its per-row top-k_cap candidates, the 65536-bin histogram of
their bf16 keys is summed over the shards (exact int32 P2P all-reduce), every rank derives the
same threshold, and the per-row tie counts [S, B] are summed the same way so that ties at the
threshold are kept in (row, global latent) order on every shard.
"""

from __future__ import annotations

import os
from typing import Any

import torch
import torch.distributed as dist

from saelens_b200.parallel.profiling import nccl_nvtx_range
from saelens_b200.parallel.symm_heap import SlabBuffer, SymmetricHeap, slab_bytes_needed
from saelens_b200.training.engine import EngineStepResult, FusedTopKEngine, update_topk_threshold_ema


# decode -> reduce-scatter: one ticketed launch, or two with SAELENS_B200_DECODE_RS=split
_DECODE_RS_LAUNCHES = 2 if os.environ.get("SAELENS_B200_DECODE_RS") == "split" else 1

class _AllReduceBufs:
    """Slab areas of one two-shot P2P all-reduce of `n` elements."""

    def __init__(self, heap: SymmetricHeap, nat: Any, n: int, dtype: torch.dtype):
        esz = torch.empty((), dtype=dtype).element_size()
        land, cnt, out, flag = nat.p2p_allreduce_sizes(n, esz, heap.world)
        self.n = n
        self.land = heap.alloc_bytes(land)
        self.cnt = heap.alloc_bytes(cnt)
        self.out_buf = heap.alloc((out // esz,), dtype)
        self.flag = heap.alloc_bytes(flag)
        self.out = heap.local(self.out_buf)[:n]

    @staticmethod
    def nbytes(nat: Any, n: int, esz: int, world: int) -> list[int]:
        return list(nat.p2p_allreduce_sizes(n, esz, world))


class _FusedBufs:
    """Peer-memory buffers of the fused TP step for one batch size (main or aux exchanges)."""

    def __init__(self, group: dist.ProcessGroup, nat: Any, B: int, D: int, k: int, world: int,
                 with_input: bool, batch_topk: bool = False):
        Bo = B // world
        f4, i4, b2 = 4, 4, 2
        sizes = []
        if with_input:
            sizes += [B * D * b2, (B // 128) * 4]
        sizes += [world * B * k * f4, world * B * k * i4, (B // 16) * 4,   # candidates
                  world * Bo * D * f4, (Bo // 16) * 4, B * D * b2, (B // 16) * 4]  # decode
        if with_input:
            sizes += _AllReduceBufs.nbytes(nat, 2 * D + 3, 4, world) + _AllReduceBufs.nbytes(nat, 1, 4, world)
        if batch_topk:
            sizes += _AllReduceBufs.nbytes(nat, 65536, 4, world) + _AllReduceBufs.nbytes(nat, world * B, 4, world)
        heap = SymmetricHeap(group, slab_bytes_needed(sizes) + 4096)
        self.heap = heap
        self.B, self.Bo, self.k = B, Bo, k
        if with_input:
            self.x: SlabBuffer | None = heap.alloc((B, D), torch.bfloat16)
            self.ag_flags = heap.alloc(B // 128, torch.int32)
        else:
            self.x = None
        self.cv = heap.alloc((world, B, k), torch.float32)
        self.ci = heap.alloc((world, B, k), torch.int32)
        self.ccnt = heap.alloc(B // 16, torch.int32)
        self.land = heap.alloc((world, Bo, D), torch.float32)
        self.lcnt = heap.alloc(Bo // 16, torch.int32)
        self.dx = heap.alloc((B, D), torch.bfloat16)
        self.dcnt = heap.alloc(B // 16, torch.int32)
        self.dx_local = heap.local(self.dx)
        self.dcnt_local = heap.local(self.dcnt)
        self.x_local = heap.local(self.x) if self.x is not None else None
        if with_input:
            self.red = _AllReduceBufs(heap, nat, 2 * D + 3, torch.float32)
            self.dead = _AllReduceBufs(heap, nat, 1, torch.float32)
        if batch_topk:  # BatchTopK: summed key histogram and per-(rank, row) tie counts
            self.hist = _AllReduceBufs(heap, nat, 65536, torch.int32)
            self.ties = _AllReduceBufs(heap, nat, world * B, torch.int32)
        self.epochs: dict[str, int] = {}

    def next_epoch(self, name: str) -> int:
        e = self.epochs.get(name, 0) + 1
        self.epochs[name] = e
        return e

    def close(self) -> None:
        self.heap.close()


class _DPReducer:
    """Averages a TP rank's latent-shard gradients over the data-parallel replicas of that shard
    (the ranks of `group` hold the same latents and see different rows) with the P2P all-reduce
    kernel, and sums the firing counts.  Gradient rows are dense ([2, N, D] buffer, zero rows for
    latents no local pair touched) because other replicas may touch them.  The rows are reduced
    in `segments` latent ranges on a communication stream while the next range's gradients are
    computed (the overlap of the DDP engine)."""

    def __init__(self, eng: "TPTopKEngine", group: dist.ProcessGroup, small_n: int, segments: int = 4):
        from saelens_b200.parallel.ddp_engine import _ArArea

        nat, N, D = eng.native, eng.N, eng.D
        self.size = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        segments = max(1, min(int(segments), N // 256))
        bounds = [N * i // segments // 256 * 256 for i in range(segments)] + [N]
        self.ranges = [(bounds[i], bounds[i + 1]) for i in range(segments) if bounds[i + 1] > bounds[i]]
        sizes = [2 * N * D * 2]
        for j0, j1 in self.ranges:
            sizes += _ArArea.nbytes(nat, (j1 - j0) * D, 2, self.size, False) * 2
        sizes += _ArArea.nbytes(nat, small_n, 4, self.size, True) + _ArArea.nbytes(nat, N, 4, self.size, True)
        self.heap = SymmetricHeap(group, slab_bytes_needed(sizes) + 65536)
        self.gbuf = torch.empty(2, N, D, dtype=torch.bfloat16, device=eng.device)
        self.gout_buf = self.heap.alloc((2, N, D), torch.bfloat16)
        self.g_avg = self.heap.local(self.gout_buf)
        base = self.gout_buf.offset
        self.areas = [(j0, j1, _ArArea(self.heap, nat, (j1 - j0) * D, 2, base + j0 * D * 2),
                       _ArArea(self.heap, nat, (j1 - j0) * D, 2, base + (N + j0) * D * 2)) for j0, j1 in self.ranges]
        self.a_small = _ArArea(self.heap, nat, small_n, 4, None)
        self.a_fire = _ArArea(self.heap, nat, N, 4, None)
        self.small_out = self.heap.local(SlabBuffer(self.a_small.out, (small_n,), torch.float32))
        self.fire_out = self.heap.local(SlabBuffer(self.a_fire.out, (N,), torch.float32))
        self.tickets = torch.zeros(2 * len(self.areas) + 2, dtype=torch.int32, device=eng.device)
        self.dense_colptr = torch.arange(N + 1, dtype=torch.int64, device=eng.device)
        self.comm = torch.cuda.Stream(device=eng.device)
        self.nat, self.status = nat, eng.status

    def _ar(self, x: torch.Tensor, scale: float, area: Any, t: int, sq: bool) -> None:
        area.epoch += 1
        self.nat.p2p_allreduce(x, scale, self.heap.bases, self.rank, area.land, area.cnt, area.out, area.flag,
                               area.epoch, self.tickets[t : t + 1], self.status.tensor,
                               area.sq_buf.offset if sq else -1)

    def reduce_segment(self, i: int) -> None:
        """Average segment i's gradient rows on the communication stream (after the compute
        stream's work so far)."""
        j0, j1, a_dec, a_enc = self.areas[i]
        ready = torch.cuda.Event()
        ready.record()
        with torch.cuda.stream(self.comm):
            self.comm.wait_event(ready)
            inv = 1.0 / self.size
            self._ar(self.gbuf[0, j0:j1].reshape(-1), inv, a_dec, 2 * i, True)
            self._ar(self.gbuf[1, j0:j1].reshape(-1), inv, a_enc, 2 * i + 1, True)

    def finish(self, small: torch.Tensor, fire: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
        """Returns (averaged small vector, summed fire counts, sum of squares of the averaged W
        grads); the compute stream waits for every reduction."""
        nt = 2 * len(self.areas)
        ready = torch.cuda.Event()
        ready.record()
        with torch.cuda.stream(self.comm):
            self.comm.wait_event(ready)
            self._ar(small, 1.0 / self.size, self.a_small, nt, False)
            self._ar(fire, 1.0, self.a_fire, nt + 1, False)
        done = torch.cuda.Event()
        done.record(self.comm)
        torch.cuda.current_stream().wait_event(done)
        sq = sum(a.sq.sum() + b.sq.sum() for _, _, a, b in self.areas)
        return self.small_out, self.fire_out, sq

    def close(self) -> None:
        self.heap.close()


class TPTopKEngine(FusedTopKEngine):
    def __init__(self, sae: Any, lr: float, group: dist.ProcessGroup, beta1: float = 0.9, beta2: float = 0.999,
                 eps: float = 1e-8, max_grad_norm: float = 1.0, input_layout: str = "row_sharded",
                 h_buffer_bytes: int = 8 << 30, fused: bool = True, dp_group: dist.ProcessGroup | None = None):
        if input_layout not in ("row_sharded", "replicated"):
            raise ValueError("input_layout must be 'row_sharded' or 'replicated'")
        self.group = group
        self.rank = dist.get_rank(group)
        self.size = dist.get_world_size(group)
        self.input_layout = input_layout
        super().__init__(sae, lr=lr, beta1=beta1, beta2=beta2, eps=eps, max_grad_norm=max_grad_norm,
                         h_buffer_bytes=h_buffer_bytes)
        self.n_local = self.N
        self.collectives = 0
        self.fused = bool(fused) and self.size <= 8
        self._fb: _FusedBufs | None = None
        self._fb_aux: _FusedBufs | None = None
        self._ticket = torch.zeros(4, dtype=torch.int32, device=self.device)
        # data parallel over replicas of this latent shard (tensor x data parallel)
        self._dp: _DPReducer | None = None
        if dp_group is not None and dist.get_world_size(dp_group) > 1:
            if not self.fused:
                raise NotImplementedError("tensor x data parallel needs the fused exchanges (fused=True)")
            segments = int(os.environ.get("SAELENS_B200_DP_SEGMENTS", "1"))
            self._dp = _DPReducer(self, dp_group, self.N + 2 * self.D + 2, segments)
            self.g_dec, self.g_enc = self._dp.gbuf[0], self._dp.gbuf[1]

    def close(self) -> None:
        """Release the peer-memory slabs (collective)."""
        for b in (self._fb, self._fb_aux):
            if b is not None:
                b.close()
        self._fb = self._fb_aux = None
        if self._dp is not None:
            self._dp.close()
            self._dp = None

    def _fused_bufs(self, B: int) -> _FusedBufs:
        if self._fb is None or self._fb.B != B:
            if self._fb is not None:
                self._fb.close()
            self._fb = _FusedBufs(self.group, self.native, B, self.D, self.k, self.size, with_input=True,
                                  batch_topk=self.batch_topk)
        return self._fb

    def _fused_aux_bufs(self, B: int, k_aux: int) -> _FusedBufs:
        if self._fb_aux is None or self._fb_aux.B != B:
            if self._fb_aux is not None:
                self._fb_aux.close()
            self._fb_aux = _FusedBufs(self.group, self.native, B, self.D, k_aux, self.size, with_input=False)
        return self._fb_aux

    # ------------------------------------------------------------------ helpers
    def _ag(self, out: torch.Tensor, inp: torch.Tensor, name: str) -> None:
        with nccl_nvtx_range(f"nccl:tp_{name}_all_gather", self.group):
            dist.all_gather_into_tensor(out, inp.contiguous(), group=self.group)
        self.collectives += 1

    def _local_rows(self, x: torch.Tensor) -> torch.Tensor:
        if self.input_layout == "replicated":
            B = x.shape[0]
            if B % self.size:
                raise ValueError(f"batch {B} not divisible by tp size {self.size}")
            b = B // self.size
            return x[self.rank * b : (self.rank + 1) * b]
        return x

    def _global_topk(self, vals: torch.Tensor, idx: torch.Tensor, k: int, k_dev: torch.Tensor | None) -> None:
        """Keep in (vals, idx) only this rank's entries of the global per-row top-k."""
        B = vals.shape[0]
        cv = torch.empty(self.size * B, k, dtype=torch.float32, device=self.device)
        ci = torch.empty(self.size * B, k, dtype=torch.int32, device=self.device)
        self._ag(cv, vals, "topk_candidates")
        self._ag(ci, idx, "topk_candidate_idx")
        self.native.topk_merge(cv.view(self.size, B, k), ci.view(self.size, B, k), self.n_local, self.rank,
                               k_dev, vals, idx)
        self.launches += 1

    def _batch_select(self, vals: torch.Tensor, idx: torch.Tensor, fb: _FusedBufs | None, ep: int) -> None:
        """BatchTopK over the shards (see the module docstring).  Leaves in (vals, idx) only this
        rank's entries among the round(k * B) largest of the TP batch."""
        nat, S, r, B = self.native, self.size, self.rank, vals.shape[0]
        K = int(round(self.batch_k * B))
        hist = torch.empty(65536, dtype=torch.int32, device=self.device)
        sel = torch.empty(4, dtype=torch.int32, device=self.device)
        ties = torch.zeros(S, B, dtype=torch.int32, device=self.device)
        prefix = torch.empty(B, dtype=torch.int64, device=self.device)
        nat.batch_hist(vals, idx, hist)
        if fb is not None:
            st, tk = self.status.tensor, self._ticket
            nat.p2p_allreduce(hist, 1.0, fb.heap.bases, r, fb.hist.land, fb.hist.cnt, fb.hist.out_buf.offset,
                              fb.hist.flag, ep, tk, st)
            hist = fb.hist.out
        else:
            with nccl_nvtx_range("nccl:tp_batch_hist_all_reduce", self.group):
                dist.all_reduce(hist, group=self.group)
            self.collectives += 1
        nat.batch_thresh(hist, K, sel)
        nat.batch_ties(vals, idx, sel, ties[r])
        if fb is not None:
            nat.p2p_allreduce(ties.view(-1), 1.0, fb.heap.bases, r, fb.ties.land, fb.ties.cnt,
                              fb.ties.out_buf.offset, fb.ties.flag, ep, tk, st)
            ties = fb.ties.out.view(S, B)
            self.launches += 2
        else:
            with nccl_nvtx_range("nccl:tp_batch_ties_all_reduce", self.group):
                dist.all_reduce(ties, group=self.group)
            self.collectives += 1
        nat.batch_filter(vals, idx, sel, ties, r, prefix, self.batch_truncated)
        self.launches += 5
        update_topk_threshold_ema(self.sae, sel)

    # ------------------------------------------------------------------ the step
    @torch.no_grad()
    def step(self, x: torch.Tensor, lr: float | None = None, dead_mask: torch.Tensor | None = None,
             want_sae_out: bool = False, act_freq: torch.Tensor | None = None,
             since_fired: torch.Tensor | None = None, run_aux: bool = False,
             update: bool = True) -> EngineStepResult:
        if self.fused:
            return self._step_fused(x, lr, dead_mask, want_sae_out, act_freq, since_fired, run_aux, update)
        nat, dev = self.native, self.device
        D, N, k, S = self.D, self.N, self.k, self.size
        x_own = self._local_rows(x)
        xb_own = x_own if (x_own.dtype == torch.bfloat16 and x_own.is_contiguous()) else \
            x_own.to(torch.bfloat16).contiguous()
        Bo = xb_own.shape[0]
        B = Bo * S
        self._mark("start")
        # 1. input rows of every rank
        if self.input_layout == "replicated" and x.dtype == torch.bfloat16 and x.is_contiguous():
            X = x
        else:
            X = torch.empty(B, D, dtype=torch.bfloat16, device=dev)
            self._ag(X, xb_own, "input_rows")
        self._mark("input_all_gather")

        # aux decision must be identical on every rank: reduce the dead count
        aux_on = False
        if run_aux and dead_mask is not None:
            nd = dead_mask.to(torch.bool).sum().to(torch.float32).reshape(1)
            with nccl_nvtx_range("nccl:tp_dead_count_all_reduce", self.group):
                dist.all_reduce(nd, group=self.group)
            self.collectives += 1
            num_dead_total = int(nd.item())
            aux_on = num_dead_total > 0
        k_aux = D // 2

        # 2. local encoder + local top-k
        R = self._row_chunk(B)
        H = torch.empty(min(R, B), N, dtype=torch.bfloat16, device=dev)
        cm = torch.empty(min(R, B), N // 32, dtype=torch.bfloat16, device=dev)
        tm = torch.empty(min(R, B), N // 256, dtype=torch.bfloat16, device=dev)  # 256-column tile maxima
        vals = torch.empty(B, k, dtype=torch.float32, device=dev)
        idx = torch.empty(B, k, dtype=torch.int32, device=dev)
        if aux_on:
            assert dead_mask is not None
            dm = dead_mask.to(torch.bool)
            k_aux_total = min(k_aux, num_dead_total)
            k_aux_dev = torch.tensor([k_aux_total], dtype=torch.int32, device=dev)
            aux_scale = min(num_dead_total / k_aux, 1.0)
            bits = dm.view(N // 32, 32).to(torch.int64) << torch.arange(32, device=dev, dtype=torch.int64)
            w = bits.sum(1)
            mask_words = torch.where(w >= 2**31, w - 2**32, w).to(torch.int32).contiguous()
            local_dead = min(int(dm.sum().item()), k_aux_total)
            aux_vals = torch.empty(B, k_aux, dtype=torch.float32, device=dev)
            aux_idx = torch.empty(B, k_aux, dtype=torch.int32, device=dev)
            k_loc_dev = torch.tensor([local_dead], dtype=torch.int32, device=dev)
        for r0 in range(0, B, R):
            r1 = min(B, r0 + R)
            h, c, t = H[: r1 - r0], cm[: r1 - r0], tm[: r1 - r0]
            nat.gemm_tn_bf16(X[r0:r1], self.w_enc, self.bias_eff, self.scale if self.rescale else None, False,
                             h, c, self.status.tensor, 0, tmax=t)
            self._mark("encoder_gemm")
            nat.row_topk(h, c, k, None, None, vals[r0:r1], idx[r0:r1], self.status.tensor, tmax=t)
            self._mark("row_topk")
            self.launches += 2
            if aux_on:
                nat.row_topk(h, c, k_aux, k_loc_dev, mask_words, aux_vals[r0:r1], aux_idx[r0:r1], self.status.tensor)
                self.launches += 1
        del H, cm, tm

        # 3. global top-k from the shards' candidates (BatchTopK: batch-wide threshold)
        if self.batch_topk:
            self._batch_select(vals, idx, None, 0)
        else:
            self._global_topk(vals, idx, k, None)
        if aux_on:
            self._global_topk(aux_vals, aux_idx, k_aux, k_aux_dev)
        self._mark("topk_exchange")

        # 4. partial decode -> reduce-scatter -> b_dec + MSE on owned rows
        part = torch.empty(B, D, dtype=torch.float32, device=dev)
        nat.decode_partial(vals, idx, True, self.inv_scale if self.rescale else None, self.w_dec, part)
        xsum = torch.empty(Bo, D, dtype=torch.float32, device=dev)
        with nccl_nvtx_range("nccl:tp_decode_reduce_scatter", self.group):
            dist.reduce_scatter_tensor(xsum, part, group=self.group)
        self.collectives += 1
        sae_out = torch.empty(Bo, D, dtype=torch.bfloat16, device=dev) if (want_sae_out or aux_on) else None
        resid = torch.empty(Bo, D, dtype=torch.bfloat16, device=dev) if aux_on else None
        dx_own = torch.empty(Bo, D, dtype=torch.bfloat16, device=dev)
        loss_row = torch.empty(Bo, dtype=torch.float32, device=dev)
        red = torch.zeros(2 * D + 3, dtype=torch.float32, device=dev)  # [bsum | bterm | sumsq | mse | aux]
        bsum, bterm = red[:D], red[D : 2 * D]
        nat.finish_mse(xsum, self.p_bdec, xb_own, sae_out, resid, dx_own, None, 2.0 / B, loss_row, bsum)
        self.launches += 2
        self._mark("decode_reduce_scatter_mse")
        dX = torch.empty(B, D, dtype=torch.bfloat16, device=dev)
        self._ag(dX, dx_own, "dxhat")

        daux = None
        if aux_on:
            assert resid is not None
            part.zero_()
            nat.decode_partial(aux_vals, aux_idx, False, self.inv_scale if self.rescale else None, self.w_dec, part)
            asum = torch.empty(Bo, D, dtype=torch.float32, device=dev)
            with nccl_nvtx_range("nccl:tp_aux_decode_reduce_scatter", self.group):
                dist.reduce_scatter_tensor(asum, part, group=self.group)
            self.collectives += 1
            da_own = torch.empty(Bo, D, dtype=torch.bfloat16, device=dev)
            aux_row = torch.empty(Bo, dtype=torch.float32, device=dev)
            nat.finish_mse(asum, None, resid, None, None, da_own, None, 2.0 * self.aux_coef * aux_scale / B,
                           aux_row, None)
            self.launches += 2
            red[2 * D + 2] = aux_row.sum()
            daux = torch.empty(B, D, dtype=torch.bfloat16, device=dev)
            self._ag(daux, da_own, "aux_grad")
        del part

        # 5. CSC + local latent gradients
        self.counts.zero_()
        self.fire_counts.zero_()
        self.cursor.zero_()
        nat.csc_count(vals, idx, aux_vals if aux_on else None, aux_idx if aux_on else None, self.counts,
                      self.fire_counts)
        torch.cumsum(self.counts, 0, out=self.colptr[1:])
        pairs = torch.empty(B * k + (B * k_aux if aux_on else 0), dtype=torch.int64, device=dev)
        nat.csc_fill(vals, idx, aux_vals if aux_on else None, aux_idx if aux_on else None, self.colptr,
                     self.cursor, pairs)
        self._mark("csc_build")
        sumsq = red[2 * D : 2 * D + 1]
        nat.latent_grad(self.colptr, pairs, vals, aux_vals if aux_on else None,
                        self.inv_scale if self.rescale else None, dX, daux, X,
                        self.p_bdec if self.apply_b_dec else None, self.w_dec, self.w_enc, self.g_dec, self.g_enc,
                        self.g_benc, bterm if self.apply_b_dec else None, sumsq, self.fire_counts, act_freq,
                        since_fired, idx, aux_idx if aux_on else None)
        self.launches += 3
        self._mark("latent_grad")

        # 6. one all-reduce for b_dec grad terms, grad norm and losses
        red[2 * D + 1] = loss_row.sum()
        with nccl_nvtx_range("nccl:tp_grad_terms_all_reduce", self.group):
            dist.all_reduce(red, group=self.group)
        self.collectives += 1
        self._mark("grad_all_reduce")
        mse = red[2 * D + 1] / B
        aux_loss = (self.aux_coef * aux_scale * red[2 * D + 2] / B) if aux_on else torch.zeros((), device=dev)
        if update:
            self.step_count += 1
            cur_lr = self.lr if lr is None else lr
            sq = red[2 * D : 2 * D + 1]
            nat.adam_bdec(bsum, bterm if self.apply_b_dec else None, self.g_bdec, sq, self.clip, self.p_bdec,
                          self.m_bdec, self.v_bdec, cur_lr, self.beta1, self.beta2, self.eps, self.step_count,
                          self.max_grad_norm, True)
            nat.adam_rows(self.p_dec, self.m_dec, self.v_dec, self.p_enc, self.m_enc, self.v_enc, self.w_dec,
                          self.w_enc, self.g_dec, self.g_enc, self.p_benc, self.m_benc, self.v_benc, self.g_benc,
                          self.colptr, self.clip, self.p_bdec if self.apply_b_dec else None, self.scale,
                          self.inv_scale, self.bias_eff, cur_lr, self.beta1, self.beta2, self.eps, self.step_count,
                          True)
            self.launches += 2
            self.sumsq = sq
            self._mark("adam")
        self.last_loss = mse + aux_loss
        return EngineStepResult(loss=mse + aux_loss, mse_loss=mse, aux_loss=aux_loss, sae_out=sae_out,
                                topk_vals=vals, topk_idx=idx, fire_counts=self.fire_counts)

    # ------------------------------------------------------------------ fused (peer-memory) step
    def _step_fused(self, x: torch.Tensor, lr: float | None, dead_mask: torch.Tensor | None, want_sae_out: bool,
                    act_freq: torch.Tensor | None, since_fired: torch.Tensor | None, run_aux: bool,
                    update: bool) -> EngineStepResult:
        nat, dev = self.native, self.device
        D, N, k, S, r = self.D, self.N, self.k, self.size, self.rank
        st, tk = self.status.tensor, self._ticket
        x_own = self._local_rows(x)
        xb_own = x_own if (x_own.dtype == torch.bfloat16 and x_own.is_contiguous()) else \
            x_own.to(torch.bfloat16).contiguous()
        Bo = xb_own.shape[0]
        B = Bo * S
        if Bo % 128:
            raise ValueError(f"fused TP step needs a per-rank batch that is a multiple of 128, got {Bo}")
        fb = self._fused_bufs(B)
        bases = fb.heap.bases
        ep = fb.next_epoch("main")
        self._mark("start")

        aux_on = False
        k_aux = D // 2
        if run_aux and dead_mask is not None:
            nd = dead_mask.to(torch.bool).sum().to(torch.float32).reshape(1)
            nat.p2p_allreduce(nd, 1.0, bases, r, fb.dead.land, fb.dead.cnt, fb.dead.out_buf.offset, fb.dead.flag,
                              fb.next_epoch("dead"), tk, st)
            self.launches += 1
            num_dead_total = int(fb.dead.out.item())
            aux_on = num_dead_total > 0

        # 1-2. all-gather fused encoder GEMM + local top-k
        R = self._row_chunk(B)
        H = torch.empty(min(R, B), N, dtype=torch.bfloat16, device=dev)
        cm = torch.empty(min(R, B), N // 32, dtype=torch.bfloat16, device=dev)
        tm = torch.empty(min(R, B), N // 256, dtype=torch.bfloat16, device=dev)  # 256-column tile maxima
        vals = torch.empty(B, k, dtype=torch.float32, device=dev)
        idx = torch.empty(B, k, dtype=torch.int32, device=dev)
        if aux_on:
            assert dead_mask is not None
            dm = dead_mask.to(torch.bool)
            k_aux_total = min(k_aux, num_dead_total)
            k_aux_dev = torch.tensor([k_aux_total], dtype=torch.int32, device=dev)
            aux_scale = min(num_dead_total / k_aux, 1.0)
            bits = dm.view(N // 32, 32).to(torch.int64) << torch.arange(32, device=dev, dtype=torch.int64)
            w = bits.sum(1)
            mask_words = torch.where(w >= 2**31, w - 2**32, w).to(torch.int32).contiguous()
            local_dead = min(int(dm.sum().item()), k_aux_total)
            aux_vals = torch.empty(B, k_aux, dtype=torch.float32, device=dev)
            aux_idx = torch.empty(B, k_aux, dtype=torch.int32, device=dev)
            k_loc_dev = torch.tensor([local_dead], dtype=torch.int32, device=dev)
        assert fb.x is not None
        for r0 in range(0, B, R):
            r1 = min(B, r0 + R)
            h, c, t = H[: r1 - r0], cm[: r1 - r0], tm[: r1 - r0]
            nat.gemm_ag_tn_bf16(xb_own, bases, r, fb.x.offset, fb.ag_flags.offset, B, r0, r1 - r0, r0 == 0, ep,
                                self.w_enc, self.bias_eff, self.scale if self.rescale else None, False, h, c, st,
                                tk, 0, tmax=t)
            self._mark("ag_encoder_gemm")
            nat.row_topk(h, c, k, None, None, vals[r0:r1], idx[r0:r1], st, tmax=t)
            self._mark("row_topk")
            self.launches += 2
            if aux_on:
                nat.row_topk(h, c, k_aux, k_loc_dev, mask_words, aux_vals[r0:r1], aux_idx[r0:r1], st)
                self.launches += 1
        del H, cm, tm
        X = fb.x_local

        # 3. candidate all-gather fused with the global merge (BatchTopK: batch-wide threshold)
        if self.batch_topk:
            self._batch_select(vals, idx, fb, ep)
        else:
            nat.topk_exchange_merge(vals, idx, self.n_local, None, bases, r, fb.cv.offset, fb.ci.offset,
                                    fb.ccnt.offset, ep, tk, st)
            self.launches += 1
        if aux_on:
            fa = self._fused_aux_bufs(B, k_aux)
            ep_aux = fa.next_epoch("aux")
            nat.topk_exchange_merge(aux_vals, aux_idx, self.n_local, k_aux_dev, fa.heap.bases, r, fa.cv.offset,
                                    fa.ci.offset, fa.ccnt.offset, ep_aux, tk, st)
            self.launches += 1
        self._mark("topk_exchange_merge")

        # 4. decode fused with the reduce-scatter, b_dec, MSE and the dL/dx_hat all-gather
        sae_out = torch.empty(Bo, D, dtype=torch.bfloat16, device=dev) if (want_sae_out or aux_on) else None
        resid = torch.empty(Bo, D, dtype=torch.bfloat16, device=dev) if aux_on else None
        loss_row = torch.empty(Bo, dtype=torch.float32, device=dev)
        red = torch.zeros(2 * D + 3, dtype=torch.float32, device=dev)  # [bsum | bterm | sumsq | mse | aux]
        bsum, bterm = red[:D], red[D : 2 * D]
        nat.decode_rs(vals, idx, True, self.inv_scale if self.rescale else None, self.w_dec, bases, r,
                      fb.land.offset, fb.lcnt.offset, fb.dx.offset, fb.dcnt.offset, ep, self.p_bdec, xb_own,
                      sae_out, resid, None, 2.0 / B, loss_row, bsum, tk, st)
        self.launches += _DECODE_RS_LAUNCHES
        daux = None
        if aux_on:
            assert resid is not None
            aux_row = torch.empty(Bo, dtype=torch.float32, device=dev)
            nat.decode_rs(aux_vals, aux_idx, False, self.inv_scale if self.rescale else None, self.w_dec,
                          fa.heap.bases, r, fa.land.offset, fa.lcnt.offset, fa.dx.offset, fa.dcnt.offset, ep_aux,
                          None, resid, None, None, None, 2.0 * self.aux_coef * aux_scale / B, aux_row, None, tk, st)
            self.launches += _DECODE_RS_LAUNCHES
            red[2 * D + 2] = aux_row.sum()
            daux = fa.dx_local
        self._mark("decode_reduce_scatter_mse")

        # 5. CSC + local latent gradients (after every rank's dL/dx_hat rows arrived)
        nat.p2p_wait_flags(fb.dcnt_local, ep, st)
        self.launches += 1
        if aux_on:
            nat.p2p_wait_flags(fa.dcnt_local, ep_aux, st)
            self.launches += 1
        dX = fb.dx_local
        self.counts.zero_()
        self.fire_counts.zero_()
        self.cursor.zero_()
        nat.csc_count(vals, idx, aux_vals if aux_on else None, aux_idx if aux_on else None, self.counts,
                      self.fire_counts)
        torch.cumsum(self.counts, 0, out=self.colptr[1:])
        pairs = torch.empty(B * k + (B * k_aux if aux_on else 0), dtype=torch.int64, device=dev)
        nat.csc_fill(vals, idx, aux_vals if aux_on else None, aux_idx if aux_on else None, self.colptr,
                     self.cursor, pairs)
        self._mark("csc_build")
        sumsq = red[2 * D : 2 * D + 1]
        dp = self._dp
        if dp is None:
            nat.latent_grad(self.colptr, pairs, vals, aux_vals if aux_on else None,
                            self.inv_scale if self.rescale else None, dX, daux, X,
                            self.p_bdec if self.apply_b_dec else None, self.w_dec, self.w_enc, self.g_dec,
                            self.g_enc, self.g_benc, bterm if self.apply_b_dec else None, sumsq, self.fire_counts,
                            act_freq, since_fired, idx, aux_idx if aux_on else None, 0, -1, False)
            self.launches += 3
        else:
            # dense rows by latent range; each range is averaged over the replicas on the
            # communication stream while the next range's gradients are computed
            for i, (j0, j1, _, _) in enumerate(dp.areas):
                nat.latent_grad(self.colptr, pairs, vals, aux_vals if aux_on else None,
                                self.inv_scale if self.rescale else None, dX, daux, X,
                                self.p_bdec if self.apply_b_dec else None, self.w_dec, self.w_enc, self.g_dec,
                                self.g_enc, self.g_benc, bterm if self.apply_b_dec else None, None, None, None, None,
                                idx, aux_idx if aux_on else None, j0, j1, True)
                dp.reduce_segment(i)
                self.launches += 5
        self._mark("latent_grad")
        red[2 * D + 1] = loss_row.sum()
        g_dec, g_enc, g_benc, colptr = self.g_dec, self.g_enc, self.g_benc, self.colptr
        if dp is not None:
            # average this shard's gradients over its data-parallel replicas; the clip norm is taken
            # from the averaged gradients (then summed over the tensor-parallel shards below)
            small = torch.cat([self.g_benc, red[: 2 * D], red[2 * D + 1 : 2 * D + 3]])
            avg, fired, sq_w = dp.finish(small, self.fire_counts.to(torch.float32))
            self.launches += 2
            N = self.N
            g_benc = avg[:N]
            red = torch.cat([avg[N : N + 2 * D], (sq_w + g_benc.square().sum()).reshape(1), avg[N + 2 * D :]])
            g_dec, g_enc, colptr = dp.g_avg[0], dp.g_avg[1], dp.dense_colptr
            if act_freq is not None:
                act_freq += fired
            if since_fired is not None:
                since_fired.copy_(torch.where(fired > 0, torch.zeros_like(since_fired), since_fired + 1))
            self.fire_counts.copy_(fired.round().to(torch.int32))
            self._mark("dp_grad_all_reduce")

        # 6. one P2P all-reduce for b_dec grad terms, grad norm and losses
        nat.p2p_allreduce(red, 1.0, bases, r, fb.red.land, fb.red.cnt, fb.red.out_buf.offset, fb.red.flag, ep,
                          tk, st)
        self.launches += 1
        red = fb.red.out
        self._mark("grad_all_reduce")
        mse = red[2 * D + 1] / B
        aux_loss = (self.aux_coef * aux_scale * red[2 * D + 2] / B) if aux_on else torch.zeros((), device=dev)
        if update:
            self.step_count += 1
            cur_lr = self.lr if lr is None else lr
            sq = red[2 * D : 2 * D + 1]
            nat.adam_bdec(red[:D], red[D : 2 * D] if self.apply_b_dec else None, self.g_bdec, sq, self.clip,
                          self.p_bdec, self.m_bdec, self.v_bdec, cur_lr, self.beta1, self.beta2, self.eps,
                          self.step_count, self.max_grad_norm, True)
            nat.adam_rows(self.p_dec, self.m_dec, self.v_dec, self.p_enc, self.m_enc, self.v_enc, self.w_dec,
                          self.w_enc, g_dec, g_enc, self.p_benc, self.m_benc, self.v_benc, g_benc.contiguous(),
                          colptr, self.clip, self.p_bdec if self.apply_b_dec else None, self.scale,
                          self.inv_scale, self.bias_eff, cur_lr, self.beta1, self.beta2, self.eps, self.step_count,
                          True)
            self.launches += 2
            self.sumsq = sq.clone()  # the slab area is rewritten by the next step
            self._mark("adam")
        self.last_loss = mse + aux_loss
        return EngineStepResult(loss=mse + aux_loss, mse_loss=mse, aux_loss=aux_loss, sae_out=sae_out,
                                topk_vals=vals, topk_idx=idx, fire_counts=self.fire_counts)
