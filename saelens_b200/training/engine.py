"""Fused native training step for TopK-family SAEs on B200.

One `FusedTopKEngine.step(x)` performs what the reference does with autograd over dense
[batch, d_sae] tensors (sae_lens/saes/topk_sae.py:615-813, sae_lens/training/sae_trainer.py:
595-780) as a fixed sequence of sm_100a kernels:

  1. tcgen05 encoder GEMM  H = bf16(((x W_enc) + b_enc - W_enc^T b_dec) * ||W_dec||) + chunk maxima
  2. exact row top-k over H, pruned by the chunk maxima           -> (value, index) x k per row
  3. sparse k-active decode + MSE + dL/dx_hat (+ column sum for the b_dec gradient)
  4. (dead latents present) masked top-k_aux, aux decode against the residual
  5. latent-major (CSC) pair lists
  6. per-latent gradients of W_dec, W_enc, b_enc + firing statistics + squared grad norm
  7. b_dec gradient, clip coefficient (on device), Adam on b_dec
  8. row-fused Adam on W_dec / W_enc / b_enc that also emits the next step's ||W_dec|| and
     folded encoder bias

State: fp32 master weights, fp32 Adam moments and bf16 compute copies, all latent-major
([d_sae, d_in]).  The SAE module's parameters are replaced by views of the fp32 masters so
that no second copy of the weights exists; `sync_module()` is therefore a no-op for the
weights.  Nothing in a step reads a value back to the host, except the number of dead latents
once `dead_feature_window` steps have passed (the aux loss needs to know whether to run).
"""

from __future__ import annotations

import math
import os
from dataclasses import dataclass
from typing import Any

import torch
from torch import nn

from saelens_b200 import ops
from saelens_b200.ops.status import StatusWord


@dataclass
class EngineStepResult:
    loss: torch.Tensor          # scalar fp32 on device (mse + aux)
    mse_loss: torch.Tensor      # scalar fp32 on device
    aux_loss: torch.Tensor      # scalar fp32 on device
    sae_out: torch.Tensor | None  # [B, d_in] bf16 reconstruction (if requested)
    topk_vals: torch.Tensor     # [B, k] fp32 pre-activations of the selected latents (pre-ReLU)
    topk_idx: torch.Tensor      # [B, k] int32 selected latent indices (-1 = none)
    fire_counts: torch.Tensor   # [d_sae] int32 rows in which each latent fired this step
    l0: torch.Tensor | None = None  # mean active latents per row, when the step keeps no per-row lists
    extra_losses: dict[str, torch.Tensor] | None = None  # further named loss terms (already in `loss`)

    def feature_acts_sparse(self, d_sae: int) -> torch.Tensor:
        """Sparse COO [B, d_sae] of ReLU'd activations (what the reference's TopK emits)."""
        if self.topk_idx is None:
            raise RuntimeError("this native step (dense form) keeps no per-row activation lists")
        B, k = self.topk_idx.shape
        live = (self.topk_idx >= 0) & (self.topk_vals > 0)
        rows = torch.arange(B, device=self.topk_idx.device).unsqueeze(1).expand(B, k)[live]
        cols = self.topk_idx[live].long()
        vals = self.topk_vals[live]
        return torch.sparse_coo_tensor(torch.stack([rows, cols]), vals, (B, d_sae)).coalesce()


def _round_up(x: int, m: int) -> int:
    return (x + m - 1) // m * m


@dataclass
class _StepState:
    """Forward results handed from the forward half of a step to the gradient/optimizer half."""

    B: int
    xb: torch.Tensor
    vals: torch.Tensor
    idx: torch.Tensor
    aux_on: bool
    aux_vals: torch.Tensor | None
    aux_idx: torch.Tensor | None
    dxhat: torch.Tensor
    daux: torch.Tensor | None
    bsum: torch.Tensor
    pairs: torch.Tensor
    mse: torch.Tensor
    aux_loss: torch.Tensor
    sae_out: torch.Tensor | None
    act_freq: torch.Tensor | None
    since_fired: torch.Tensor | None
    lr: float | None
    update: bool


def update_topk_threshold_ema(sae: Any, sel: torch.Tensor) -> None:
    """BatchTopK inference threshold: EMA of the smallest kept activation
    (sae_lens/saes/batchtopk_sae.py:116-125).  sel[3] is that value's 16-bit order key (0 when
    nothing was kept); kept values are exact bf16, so the key gives the value exactly."""
    k3 = sel[3]
    kept = ((k3 & 0x7FFF) << 16).view(torch.float32)
    thr = sae.topk_threshold
    lr_t = float(sae.cfg.topk_threshold_lr)
    thr.copy_(torch.where(k3 > 0x8000, (1 - lr_t) * thr + lr_t * kept.to(thr.dtype), thr))


class FusedTopKEngine:
    """Owns the optimizer state of a (possibly latent-sharded) TopK SAE and steps it natively."""

    def __init__(self, sae: Any, lr: float, beta1: float = 0.9, beta2: float = 0.999, eps: float = 1e-8,
                 max_grad_norm: float = 1.0, h_buffer_bytes: int = 8 << 30):
        if not torch.cuda.is_available():
            raise RuntimeError("FusedTopKEngine needs a CUDA device")
        self.native = ops.native()
        self.sae = sae
        cfg = sae.cfg
        # BatchTopK: keep the k * B largest activations of the batch.  Each row contributes its
        # top `batch_topk_cap` candidates (4k by default) to the batch-wide selection.
        from saelens_b200.models.batchtopk import BatchTopKTrainingSAE

        self.batch_topk = isinstance(sae, BatchTopKTrainingSAE)
        self.batch_k = float(getattr(cfg, "k", 0) or 0)
        if self.batch_topk:
            self.k = int(min(1024, sae.cfg.d_sae, max(1, round(4 * float(cfg.k)))))
        elif hasattr(cfg, "k"):
            self.k = int(cfg.k)
        else:  # threshold-sparse SAEs: `k` is the per-row candidate capacity
            self.k = int(min(1024, sae.cfg.d_sae))
        self.rescale = bool(getattr(cfg, "rescale_acts_by_decoder_norm", False))
        self.aux_coef = float(getattr(cfg, "aux_loss_coefficient", 1.0))
        self.apply_b_dec = bool(cfg.apply_b_dec_to_input)
        if cfg.normalize_activations in ("constant_norm_rescale", "layer_norm"):
            raise ValueError("the fused engine supports normalize_activations none / expected_average_only_in")
        self.lr, self.beta1, self.beta2, self.eps = lr, beta1, beta2, eps
        self.max_grad_norm = max_grad_norm
        self.device = sae.W_dec.device
        dev = self.device
        W_dec = sae.W_dec.detach()
        W_enc = sae.W_enc.detach()
        self.N, self.D = W_dec.shape
        self.k = min(self.k, self.N)  # a latent shard may be narrower than the candidate cap
        if self.D % 64 != 0 or self.N % 256 != 0:
            raise ValueError(f"fused engine needs d_in % 64 == 0 and local d_sae % 256 == 0, got {self.D}, {self.N}")
        if self.k > self.N:
            raise ValueError("k larger than the (local) number of latents")
        f32 = torch.float32
        # fp32 masters (latent-major) and moments
        self.p_dec = torch.empty(self.N, self.D, dtype=f32, device=dev).copy_(W_dec)
        self.p_enc = torch.empty(self.N, self.D, dtype=f32, device=dev).copy_(W_enc.T)
        self.p_benc = torch.empty(self.N, dtype=f32, device=dev).copy_(sae.b_enc.detach())
        self.p_bdec = torch.empty(self.D, dtype=f32, device=dev).copy_(sae.b_dec.detach())
        del W_dec, W_enc
        self._alias_module()  # drops the module's own copies before the large state is allocated
        self.m_dec, self.v_dec = torch.zeros_like(self.p_dec), torch.zeros_like(self.p_dec)
        self.m_enc, self.v_enc = torch.zeros_like(self.p_enc), torch.zeros_like(self.p_enc)
        self.m_benc, self.v_benc = torch.zeros_like(self.p_benc), torch.zeros_like(self.p_benc)
        self.m_bdec, self.v_bdec = torch.zeros_like(self.p_bdec), torch.zeros_like(self.p_bdec)
        # bf16 compute copies, gradients, per-latent vectors for the next forward
        bf = torch.bfloat16
        self.w_dec = torch.empty(self.N, self.D, dtype=bf, device=dev)
        self.w_enc = torch.empty(self.N, self.D, dtype=bf, device=dev)
        self.g_dec = torch.empty(self.N, self.D, dtype=bf, device=dev)
        self.g_enc = torch.empty(self.N, self.D, dtype=bf, device=dev)
        self.g_benc = torch.zeros(self.N, dtype=f32, device=dev)
        self.g_bdec = torch.zeros(self.D, dtype=f32, device=dev)
        self.scale = torch.empty(self.N, dtype=f32, device=dev)
        self.inv_scale = torch.empty(self.N, dtype=f32, device=dev)
        self.bias_eff = torch.empty(self.N, dtype=f32, device=dev)
        self.sumsq = torch.zeros(1, dtype=f32, device=dev)
        self.clip = torch.ones(1, dtype=f32, device=dev)
        self.counts = torch.zeros(self.N, dtype=torch.int32, device=dev)
        self.fire_counts = torch.zeros(self.N, dtype=torch.int32, device=dev)
        self.cursor = torch.zeros(self.N, dtype=torch.int32, device=dev)
        self.colptr = torch.zeros(self.N + 1, dtype=torch.int64, device=dev)
        self.status = StatusWord(dev)
        self.batch_truncated = torch.zeros(1, dtype=torch.int32, device=dev)  # rows whose candidate cap was hit
        self.h_buffer_bytes = h_buffer_bytes
        self.step_count = 0  # Adam steps taken
        self.launches = 0    # native kernel launches issued by step() so far
        self.last_loss: torch.Tensor | None = None
        # per-phase CUDA-event timing (SAELENS_B200_PHASE_TIMING=1); read with phase_times_ms()
        self._phase_timing = os.environ.get("SAELENS_B200_PHASE_TIMING", "0") == "1"
        self._phase_events: list[tuple[str, torch.cuda.Event]] = []
        self._phase_acc: dict[str, float] = {}
        self.refresh()

    # ------------------------------------------------------------------ state plumbing
    def _alias_module(self) -> None:
        """Point the module's parameters at the fp32 masters (no duplicate weight storage)."""
        sae = self.sae
        sae.W_dec = nn.Parameter(self.p_dec, requires_grad=False)
        sae.W_enc = nn.Parameter(self.p_enc.T, requires_grad=False)
        sae.b_enc = nn.Parameter(self.p_benc, requires_grad=False)
        sae.b_dec = nn.Parameter(self.p_bdec, requires_grad=False)
        sae.dtype = torch.float32

    def refresh(self) -> None:
        """Recompute bf16 copies, ||W_dec|| and the folded bias from the fp32 masters."""
        self.native.adam_rows(
            self.p_dec, self.m_dec, self.v_dec, self.p_enc, self.m_enc, self.v_enc, self.w_dec, self.w_enc,
            None, None, self.p_benc, self.m_benc, self.v_benc, None, None, None,
            self.p_bdec if self.apply_b_dec else None, self.scale, self.inv_scale, self.bias_eff,
            self.lr, self.beta1, self.beta2, self.eps, 1, False,
        )

    def optimizer_state(self) -> dict[str, dict[str, Any]]:
        """Named Adam state in the reference layout (W_enc moments as [d_in, d_sae])."""
        st = torch.tensor(float(self.step_count))
        return {
            "W_dec": {"step": st.clone(), "exp_avg": self.m_dec, "exp_avg_sq": self.v_dec},
            "W_enc": {"step": st.clone(), "exp_avg": self.m_enc.T, "exp_avg_sq": self.v_enc.T},
            "b_enc": {"step": st.clone(), "exp_avg": self.m_benc, "exp_avg_sq": self.v_benc},
            "b_dec": {"step": st.clone(), "exp_avg": self.m_bdec, "exp_avg_sq": self.v_bdec},
        }

    @torch.no_grad()
    def load_optimizer_state(self, state: dict[str, dict[str, Any]]) -> None:
        def cp(dst: torch.Tensor, src: torch.Tensor) -> None:
            dst.copy_(src.to(device=dst.device, dtype=dst.dtype))

        if "W_dec" in state:
            cp(self.m_dec, state["W_dec"]["exp_avg"])
            cp(self.v_dec, state["W_dec"]["exp_avg_sq"])
            self.step_count = int(float(state["W_dec"].get("step", self.step_count)))
        if "W_enc" in state:
            cp(self.m_enc, state["W_enc"]["exp_avg"].T)
            cp(self.v_enc, state["W_enc"]["exp_avg_sq"].T)
        for name, m, v in (("b_enc", self.m_benc, self.v_benc), ("b_dec", self.m_bdec, self.v_bdec)):
            if name in state:
                cp(m, state[name]["exp_avg"])
                cp(v, state[name]["exp_avg_sq"])

    @torch.no_grad()
    def load_weights(self, W_enc: torch.Tensor, W_dec: torch.Tensor, b_enc: torch.Tensor,
                     b_dec: torch.Tensor) -> None:
        self.p_dec.copy_(W_dec)
        self.p_enc.copy_(W_enc.T)
        self.p_benc.copy_(b_enc)
        self.p_bdec.copy_(b_dec)
        self.refresh()

    def close(self) -> None:
        """Release resources shared with other ranks (none on one GPU)."""

    def _mark(self, name: str) -> None:
        if self._phase_timing:
            ev = torch.cuda.Event(enable_timing=True)
            ev.record()
            self._phase_events.append((name, ev))

    def _flush_phases(self) -> None:
        if not self._phase_events:
            return
        torch.cuda.synchronize()
        for (_, a), (name, b) in zip(self._phase_events[:-1], self._phase_events[1:]):
            self._phase_acc[name] = self._phase_acc.get(name, 0.0) + a.elapsed_time(b)
        self._phase_events.clear()

    def phase_times_ms(self, reset: bool = True) -> dict[str, float]:
        """Accumulated milliseconds per phase since the last reset (phase timing mode only)."""
        self._flush_phases()
        out = dict(self._phase_acc)
        if reset:
            self._phase_acc.clear()
        return out

    def _row_chunk(self, B: int) -> int:
        rows = max(128, (self.h_buffer_bytes // (2 * self.N)) // 128 * 128)
        return min(_round_up(B, 128), rows)

    # ------------------------------------------------------------------ the step
    @torch.no_grad()
    def step(self, x: torch.Tensor, lr: float | None = None, dead_mask: torch.Tensor | None = None,
             want_sae_out: bool = False, act_freq: torch.Tensor | None = None,
             since_fired: torch.Tensor | None = None, run_aux: bool = False,
             update: bool = True) -> EngineStepResult:
        """One training step on a batch `x` [B, d_in] already on this device.

        `act_freq` / `since_fired` (fp32 [d_sae]) are updated in place with this step's firing
        statistics (`+= fired rows` and `0 if fired else +1`).  With `run_aux` the dead-latent
        aux-k loss is computed for latents where `dead_mask` is true.
        """
        fw = self._encode_select(x, dead_mask, run_aux)
        nat, dev = self.native, self.device
        B, D, k = fw["B"], self.D, self.k
        xb, vals, idx, aux_on = fw["xb"], fw["vals"], fw["idx"], fw["aux_on"]
        aux_vals, aux_idx, aux_scale = fw.get("aux_vals"), fw.get("aux_idx"), fw.get("aux_scale")
        k_aux = D // 2

        # 3. decode + MSE + dL/dx_hat (+ sum over rows for the b_dec gradient)
        sae_out = torch.empty(B, D, dtype=torch.bfloat16, device=dev) if (want_sae_out or aux_on) else None
        dxhat = torch.empty(B, D, dtype=torch.bfloat16, device=dev)
        loss_row = torch.empty(B, dtype=torch.float32, device=dev)
        bsum = torch.zeros(D, dtype=torch.float32, device=dev)
        resid = torch.empty(B, D, dtype=torch.bfloat16, device=dev) if aux_on else None
        nat.decode_mse(vals, idx, True, self.inv_scale if self.rescale else None, self.w_dec, self.p_bdec, xb,
                       sae_out, resid, dxhat, None, 2.0 / B, loss_row, bsum)
        mse = loss_row.sum() / B
        self.launches += 1
        self._mark("decode_mse")
        daux, aux_loss = self._aux_decode(fw, resid)
        pairs = self._build_csc(fw)
        return self._grads_and_update(_StepState(
            B=B, xb=xb, vals=vals, idx=idx, aux_on=aux_on, aux_vals=aux_vals if aux_on else None,
            aux_idx=aux_idx if aux_on else None, dxhat=dxhat, daux=daux, bsum=bsum, pairs=pairs, mse=mse,
            aux_loss=aux_loss, sae_out=sae_out, act_freq=act_freq, since_fired=since_fired, lr=lr, update=update))

    def _aux_decode(self, fw: dict[str, Any], resid: torch.Tensor | None) -> tuple[torch.Tensor | None, torch.Tensor]:
        """Aux-k loss on dead latents against the residual `resid` (step 4); (dL/dx_aux, loss)."""
        nat, dev, B, D = self.native, self.device, fw["B"], self.D
        aux_loss = torch.zeros((), dtype=torch.float32, device=dev)
        if not fw["aux_on"]:
            return None, aux_loss
        daux = torch.empty(B, D, dtype=torch.bfloat16, device=dev)
        aux_row = torch.empty(B, dtype=torch.float32, device=dev)
        gcoef = (fw["aux_scale"] * (2.0 * self.aux_coef / B)).reshape(1).contiguous()
        nat.decode_mse(fw["aux_vals"], fw["aux_idx"], False, self.inv_scale if self.rescale else None, self.w_dec,
                       None, resid, None, None, daux, gcoef, 1.0, aux_row, None)
        aux_loss = self.aux_coef * fw["aux_scale"] * aux_row.sum() / B
        self.launches += 1
        return daux, aux_loss

    def _build_csc(self, fw: dict[str, Any]) -> torch.Tensor:
        """CSC pair lists of the main (and aux) selections (step 5)."""
        nat, dev, B, k = self.native, self.device, fw["B"], self.k
        aux_on = fw["aux_on"]
        self.counts.zero_()
        self.fire_counts.zero_()
        self.cursor.zero_()
        nat.csc_count(fw["vals"], fw["idx"], fw.get("aux_vals"), fw.get("aux_idx"), self.counts, self.fire_counts)
        torch.cumsum(self.counts, 0, out=self.colptr[1:])
        n_pairs = B * k + (B * (self.D // 2) if aux_on else 0)
        pairs = torch.empty(n_pairs, dtype=torch.int64, device=dev)
        nat.csc_fill(fw["vals"], fw["idx"], fw.get("aux_vals"), fw.get("aux_idx"), self.colptr, self.cursor, pairs)
        self._mark("csc_build")
        return pairs

    def _encode_select(self, x: torch.Tensor, dead_mask: torch.Tensor | None, run_aux: bool) -> dict[str, Any]:
        """Steps 1-2: encoder GEMM with chunk maxima, row top-k (and the masked aux-k top-k), and
        the batch-wide selection for BatchTopK."""
        nat = self.native
        dev = self.device
        B = x.shape[0]
        D, N, k = self.D, self.N, self.k
        xb = x if (x.dtype == torch.bfloat16 and x.is_contiguous()) else x.to(torch.bfloat16).contiguous()

        # 1-2. encoder GEMM + chunk maxima + row top-k (row-chunked to bound the H buffer)
        self._mark("start")
        R = self._row_chunk(B)
        H = torch.empty(min(R, B), N, dtype=torch.bfloat16, device=dev)
        cm = torch.empty(min(R, B), N // 32, dtype=torch.bfloat16, device=dev)
        tm = torch.empty(min(R, B), N // 256, dtype=torch.bfloat16, device=dev)  # 256-column tile maxima
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
            words = torch.zeros(N // 32 * 32, dtype=torch.int64, device=dev)
            words[: N] = dm.to(torch.int64)
            words = (words.view(N // 32, 32) << torch.arange(32, device=dev, dtype=torch.int64)).sum(1)
            mask_words = words.to(torch.int64).bitwise_and(0xFFFFFFFF)
            mask_words = torch.where(mask_words >= 2**31, mask_words - 2**32, mask_words).to(torch.int32).contiguous()
            aux_vals = torch.empty(B, k_aux, dtype=torch.float32, device=dev)
            aux_idx = torch.empty(B, k_aux, dtype=torch.int32, device=dev)
        for r0 in range(0, B, R):
            r1 = min(B, r0 + R)
            h = H[: r1 - r0]
            c = cm[: r1 - r0]
            t = tm[: r1 - r0]
            nat.gemm_tn_bf16(xb[r0:r1], self.w_enc, self.bias_eff, self.scale if self.rescale else None, False,
                             h, c, self.status.tensor, 0, tmax=t)
            self._mark("encoder_gemm")
            nat.row_topk(h, c, k, None, None, vals[r0:r1], idx[r0:r1], self.status.tensor, tmax=t)
            self._mark("row_topk")
            self.launches += 2
            if aux_on:
                self.launches += 1
                nat.row_topk(h, c, k_aux, k_aux_dev, mask_words, aux_vals[r0:r1], aux_idx[r0:r1],
                             self.status.tensor)
        del H, cm, tm
        if self.batch_topk:
            # batch-wide selection among the per-row candidates (k * B largest ReLU activations)
            sel = nat.batch_topk_select(vals, idx, int(round(self.batch_k * B)), self.batch_truncated)
            self.launches += 5
            update_topk_threshold_ema(self.sae, sel)
            self._mark("batch_topk_select")
        fw: dict[str, Any] = {"B": B, "xb": xb, "vals": vals, "idx": idx, "aux_on": aux_on}
        if aux_on:
            fw.update(aux_vals=aux_vals, aux_idx=aux_idx, aux_scale=aux_scale)
        return fw

    def _grads_and_update(self, st: "_StepState") -> EngineStepResult:
        """Latent gradients, firing statistics, clip and Adam (steps 6-8 of the step)."""
        nat, dev, D = self.native, self.device, self.D
        self.sumsq.zero_()
        bterm = torch.zeros(D, dtype=torch.float32, device=dev)
        nat.latent_grad(self.colptr, st.pairs, st.vals, st.aux_vals, self.inv_scale if self.rescale else None,
                        st.dxhat, st.daux, st.xb, self.p_bdec if self.apply_b_dec else None, self.w_dec,
                        self.w_enc, self.g_dec, self.g_enc, self.g_benc, bterm if self.apply_b_dec else None,
                        self.sumsq, self.fire_counts, st.act_freq, st.since_fired, st.idx, st.aux_idx)
        self.launches += 3
        self._mark("latent_grad")
        if st.update:
            self._update(st, bterm)
        self.last_loss = st.mse + st.aux_loss
        if self._phase_timing and len(self._phase_events) > 64:
            self._flush_phases()
        return EngineStepResult(loss=st.mse + st.aux_loss, mse_loss=st.mse, aux_loss=st.aux_loss,
                                sae_out=st.sae_out, topk_vals=st.vals, topk_idx=st.idx,
                                fire_counts=self.fire_counts)

    def _update(self, st: "_StepState", bterm: torch.Tensor) -> None:
        """Clip + Adam on b_dec and on the latent rows (step 8)."""
        nat = self.native
        self.step_count += 1
        cur_lr = self.lr if st.lr is None else st.lr
        nat.adam_bdec(st.bsum, bterm if self.apply_b_dec else None, self.g_bdec, self.sumsq, self.clip,
                      self.p_bdec, self.m_bdec, self.v_bdec, cur_lr, self.beta1, self.beta2, self.eps,
                      self.step_count, self.max_grad_norm, True)
        nat.adam_rows(self.p_dec, self.m_dec, self.v_dec, self.p_enc, self.m_enc, self.v_enc, self.w_dec,
                      self.w_enc, self.g_dec, self.g_enc, self.p_benc, self.m_benc, self.v_benc, self.g_benc,
                      self.colptr, self.clip, self.p_bdec if self.apply_b_dec else None, self.scale,
                      self.inv_scale, self.bias_eff, cur_lr, self.beta1, self.beta2, self.eps,
                      self.step_count, True)
        self.launches += 2
        self._mark("adam")

    def grad_norm(self) -> torch.Tensor:
        return self.sumsq.sqrt()


def engine_supported(sae: Any) -> bool:
    """True when `sae` can run on the fused engine (TopK family, CUDA, native ops built)."""
    from saelens_b200.models.topk import TopKTrainingSAE

    if type(sae).__name__ != "TopKTrainingSAE" and not isinstance(sae, TopKTrainingSAE):
        return False
    from saelens_b200.models.batchtopk import BatchTopKTrainingSAE

    if type(sae) not in (TopKTrainingSAE, BatchTopKTrainingSAE):  # Matryoshka: nested-width losses
        return False
    if not sae.W_dec.is_cuda or not ops.available():
        return False
    N, D = sae.W_dec.shape
    return D % 64 == 0 and N % 256 == 0 and sae.cfg.normalize_activations in ("none", "expected_average_only_in")


def smoke_step() -> dict[str, float]:
    """Tiny end-to-end native step (used by `__graft_entry__.smoke`)."""
    from saelens_b200.models.topk import TopKTrainingSAE, TopKTrainingSAEConfig

    torch.manual_seed(0)
    sae = TopKTrainingSAE(TopKTrainingSAEConfig(d_in=256, d_sae=1024, k=16, device="cuda"))
    eng = FusedTopKEngine(sae, lr=1e-3)
    x = torch.randn(512, 256, device="cuda")
    losses = []
    for _ in range(3):
        r = eng.step(x)
        losses.append(float(r.loss))
    torch.cuda.synchronize()
    eng.status.check("smoke")
    assert all(math.isfinite(v) for v in losses), losses
    return {"loss_first": losses[0], "loss_last": losses[-1]}
