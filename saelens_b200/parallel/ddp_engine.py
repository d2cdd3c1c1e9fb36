"""Data-parallel TopK training step with the gradient all-reduce done by NVLink kernels.

Every rank holds the full SAE (replicated) and trains on its own rows.  The forward half of the
step is the single-GPU fused step (encoder GEMM, row top-k, sparse decode + MSE, CSC pair lists).
The gradient half differs:

1. Latent gradients are built in `segments` latent ranges on the compute stream, with dense rows
   (zero rows for latents that no local pair touches, since other ranks may touch them).
2. As soon as a segment's rows exist, a two-shot P2P all-reduce kernel on a communication
   stream averages them over the ranks (the 1/world scale is fused) and leaves the result in
   every rank's symmetric slab, together with the per-chunk sum of squares of the averaged
   gradient.  The next segment's gradient kernels run meanwhile, so the reduction overlaps
   the backward.
3. One fp32 all-reduce averages [gb_enc | sum dL/dx_hat | b_dec term | mse | aux], and one sums
   the per-latent fire counts.
4. Clip (from the averaged gradient's norm) and the row-fused Adam run on the averaged gradients,
   identically on every rank, so the replicas stay equal without a parameter broadcast.

This replaces the reference's DDP bucket all-reduce and manual flat all-reduce
(sae_lens/llm_sae_training_runner.py:464-485, sae_lens/training/sae_trainer.py:701-738) and the
statistics all-reduces (sae_trainer.py:608-613, 656-666, 679-684).
"""

from __future__ import annotations

from typing import Any

import torch
import torch.distributed as dist

from saelens_b200.parallel.symm_heap import SlabBuffer, SymmetricHeap, slab_bytes_needed
from saelens_b200.training.engine import EngineStepResult, FusedTopKEngine, _StepState


class _ArArea:
    """Slab offsets of one P2P all-reduce call (the output may live in a shared buffer)."""

    def __init__(self, heap: SymmetricHeap, nat: Any, n: int, esz: int, out_off: int | None):
        land, cnt, out, flag = nat.p2p_allreduce_sizes(n, esz, heap.world)
        self.n = n
        self.land = heap.alloc_bytes(land)
        self.cnt = heap.alloc_bytes(cnt)
        self.flag = heap.alloc_bytes(flag)
        self.nch = cnt // 4
        self.sq_buf = heap.alloc(self.nch, torch.float32)
        self.sq = heap.local(self.sq_buf)
        self.out = out_off if out_off is not None else heap.alloc_bytes(out)
        self.epoch = 0

    @staticmethod
    def nbytes(nat: Any, n: int, esz: int, world: int, own_out: bool) -> list[int]:
        land, cnt, out, flag = nat.p2p_allreduce_sizes(n, esz, world)
        return [land, cnt, flag, cnt] + ([out] if own_out else [])


class DDPTopKEngine(FusedTopKEngine):
    def __init__(self, sae: Any, lr: float, group: dist.ProcessGroup, beta1: float = 0.9, beta2: float = 0.999,
                 eps: float = 1e-8, max_grad_norm: float = 1.0, segments: int = 4, h_buffer_bytes: int = 8 << 30):
        super().__init__(sae, lr=lr, beta1=beta1, beta2=beta2, eps=eps, max_grad_norm=max_grad_norm,
                         h_buffer_bytes=h_buffer_bytes)
        self.group = group
        self.rank = dist.get_rank(group)
        self.size = dist.get_world_size(group)
        if self.size > 8:
            raise ValueError("the P2P all-reduce supports at most 8 ranks")
        N, D, dev = self.N, self.D, self.device
        # one [2, N, D] gradient buffer so a latent range of both matrices is two contiguous runs
        self._gbuf = torch.empty(2, N, D, dtype=torch.bfloat16, device=dev)
        self.g_dec, self.g_enc = self._gbuf[0], self._gbuf[1]
        self.dense_colptr = torch.arange(N + 1, dtype=torch.int64, device=dev)
        self.segments = max(1, min(int(segments), N))
        bounds = [N * i // self.segments for i in range(self.segments + 1)]
        self._ranges = [(bounds[i], bounds[i + 1]) for i in range(self.segments) if bounds[i + 1] > bounds[i]]
        self._small_n = N + 2 * D + 2
        nat = self.native
        sizes = [2 * N * D * 2]
        for j0, j1 in self._ranges:
            sizes += _ArArea.nbytes(nat, (j1 - j0) * D, 2, self.size, False) * 2
        sizes += _ArArea.nbytes(nat, self._small_n, 4, self.size, True)
        sizes += _ArArea.nbytes(nat, N, 4, self.size, True)
        self.heap = SymmetricHeap(group, slab_bytes_needed(sizes) + 65536)
        self._gout_buf = self.heap.alloc((2, N, D), torch.bfloat16)
        self.g_avg = self.heap.local(self._gout_buf)  # averaged gradients [2, N, D]
        base = self._gout_buf.offset
        self._areas: list[tuple[int, int, _ArArea, _ArArea]] = []
        for j0, j1 in self._ranges:
            a_dec = _ArArea(self.heap, nat, (j1 - j0) * D, 2, base + j0 * D * 2)
            a_enc = _ArArea(self.heap, nat, (j1 - j0) * D, 2, base + (N + j0) * D * 2)
            self._areas.append((j0, j1, a_dec, a_enc))
        self._a_small = _ArArea(self.heap, nat, self._small_n, 4, None)
        self._a_fire = _ArArea(self.heap, nat, N, 4, None)
        self._small_out = self.heap.local(SlabBuffer(self._a_small.out, (self._small_n,), torch.float32))
        self._fire_out = self.heap.local(SlabBuffer(self._a_fire.out, (N,), torch.float32))
        self._tickets = torch.zeros(2 * len(self._areas) + 4, dtype=torch.int32, device=dev)
        self.comm = torch.cuda.Stream(device=dev)
        self.collectives = 0

    def close(self) -> None:
        self.heap.close()

    def _ar(self, x: torch.Tensor, scale: float, area: _ArArea, ticket: int, with_sq: bool) -> None:
        area.epoch += 1
        self.native.p2p_allreduce(x, scale, self.heap.bases, self.rank, area.land, area.cnt, area.out, area.flag,
                                  area.epoch, self._tickets[ticket : ticket + 1], self.status.tensor,
                                  area.sq_buf.offset if with_sq else -1)
        self.launches += 1
        self.collectives += 1

    # ------------------------------------------------------------------ gradient half
    def _grads_and_update(self, st: _StepState) -> EngineStepResult:
        nat, dev, N, D, S = self.native, self.device, self.N, self.D, self.size
        small = torch.zeros(self._small_n, dtype=torch.float32, device=dev)  # [gb_enc|bsum|bterm|mse|aux]
        gb_enc, bterm = small[:N], small[N + D : N + 2 * D]
        compute = torch.cuda.current_stream(dev)
        for i, (j0, j1, a_dec, a_enc) in enumerate(self._areas):
            nat.latent_grad(self.colptr, st.pairs, st.vals, st.aux_vals, self.inv_scale if self.rescale else None,
                            st.dxhat, st.daux, st.xb, self.p_bdec if self.apply_b_dec else None, self.w_dec,
                            self.w_enc, self.g_dec, self.g_enc, gb_enc, bterm if self.apply_b_dec else None, None,
                            None, None, None, st.idx, st.aux_idx, j0, j1, True)
            self.launches += 3
            ready = torch.cuda.Event()
            ready.record(compute)
            with torch.cuda.stream(self.comm):
                self.comm.wait_event(ready)
                self._ar(self._gbuf[0, j0:j1].reshape(-1), 1.0 / S, a_dec, 2 * i, True)
                self._ar(self._gbuf[1, j0:j1].reshape(-1), 1.0 / S, a_enc, 2 * i + 1, True)
        self._mark("latent_grad")
        small[N : N + D] = st.bsum
        small[N + 2 * D] = st.mse
        small[N + 2 * D + 1] = st.aux_loss
        fire = self.fire_counts.to(torch.float32)
        ready = torch.cuda.Event()
        ready.record(compute)
        nt = 2 * len(self._areas)
        with torch.cuda.stream(self.comm):
            self.comm.wait_event(ready)
            self._ar(small, 1.0 / S, self._a_small, nt, False)
            self._ar(fire, 1.0, self._a_fire, nt + 1, False)
        done = torch.cuda.Event()
        done.record(self.comm)
        compute.wait_event(done)
        self._mark("grad_all_reduce")

        red = self._small_out
        fired = self._fire_out
        if st.act_freq is not None:
            st.act_freq += fired
        if st.since_fired is not None:
            st.since_fired.copy_(torch.where(fired > 0, torch.zeros_like(st.since_fired), st.since_fired + 1))
        self.fire_counts.copy_(fired.round().to(torch.int32))
        gb_avg = red[:N]
        sumsq = (sum(a.sq.sum() for _, _, a, _ in self._areas) + sum(b.sq.sum() for _, _, _, b in self._areas)
                 + gb_avg.square().sum()).reshape(1)
        self.sumsq = sumsq
        mse, aux_loss = red[N + 2 * D], red[N + 2 * D + 1]
        if st.update:
            self.step_count += 1
            cur_lr = self.lr if st.lr is None else st.lr
            nat.adam_bdec(red[N : N + D], red[N + D : N + 2 * D] if self.apply_b_dec else None, self.g_bdec, sumsq,
                          self.clip, self.p_bdec, self.m_bdec, self.v_bdec, cur_lr, self.beta1, self.beta2, self.eps,
                          self.step_count, self.max_grad_norm, True)
            nat.adam_rows(self.p_dec, self.m_dec, self.v_dec, self.p_enc, self.m_enc, self.v_enc, self.w_dec,
                          self.w_enc, self.g_avg[0], self.g_avg[1], self.p_benc, self.m_benc, self.v_benc,
                          gb_avg.contiguous(), self.dense_colptr, self.clip,
                          self.p_bdec if self.apply_b_dec else None, self.scale, self.inv_scale, self.bias_eff,
                          cur_lr, self.beta1, self.beta2, self.eps, self.step_count, True)
            self.launches += 2
            self._mark("adam")
        self.last_loss = mse + aux_loss
        return EngineStepResult(loss=mse + aux_loss, mse_loss=mse, aux_loss=aux_loss, sae_out=st.sae_out,
                                topk_vals=st.vals, topk_idx=st.idx, fire_counts=self.fire_counts)
