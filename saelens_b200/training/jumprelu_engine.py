"""Native JumpReLU training step (role of sae_lens/saes/jumprelu_sae.py:19-85 and 241-300 with the
"step" L0 loss), in two forms that compute the same step:

Dense form (while many latents are active, e.g. right after init with threshold 0.001): five
tcgen05 GEMMs, no transposes in memory (MN-major operands):
  1. H = x W_enc^T + b_eff (b_dec folded), F = H * 1[H > theta] (the gate compares the stored bf16
     H), firing counts and the number of active entries in the epilogue;
  2. x_hat = F W_dec + b_dec with the MSE, dL/dx_hat = 2 (x_hat - x) / B and its column sums
     (the b_dec gradient) in the epilogue;
  3. gW_dec = F^T dL/dx_hat (sum of squares for the clip norm in the epilogue);
  4. dL/dH = (dL/dx_hat W_dec^T) * 1[H > theta] with the rectangle-window threshold gradient
     sum_b rect((H - theta) / bw) * (-(theta / bw) dL/dF - l0_coef / (B bw)) and the b_enc gradient
     (column sums) in the epilogue;
  5. gW_enc = dL/dH^T x - g_benc (x) b_dec (the rank-1 correction for the folded b_dec).
Sparse form (once rows are sparse): `threshold_select` lists, per row, every entry above
threshold - bandwidth/2 (active entries plus the straight-through window), pruned by the chunk
maxima; the sparse decode uses the active entries only; the pair lists drive the latent
gradients and the threshold gradient of every window entry.  A row with more window entries than
the candidate cap would change the step's meaning, so the sparse form checks the cap before
decoding and runs the step in the dense form instead (and stays dense for a while).
Both forms end with the clip and the row-fused Adam as for TopK, and Adam on log_threshold
(its gradient is threshold * d/dthreshold).  The L0 coefficient comes from the trainer's
coefficient schedule (`set_coefficients`).
"""

from __future__ import annotations

import math
import warnings
from typing import Any

import torch
from torch import nn

from saelens_b200.training.engine import EngineStepResult, FusedTopKEngine


class JumpReLUEngine(FusedTopKEngine):
    aux_loss_name = "l0_loss"

    # the sparse form is tried once the mean number of active latents per row is below cap / 8,
    # checked every SPARSE_CHECK_EVERY dense steps; after a fallback to dense it waits DENSE_HOLD steps
    SPARSE_CHECK_EVERY = 20
    DENSE_HOLD = 200

    def __init__(self, sae: Any, lr: float, beta1: float = 0.9, beta2: float = 0.999, eps: float = 1e-8,
                 max_grad_norm: float = 1.0, h_buffer_bytes: int = 8 << 30, cap: int = 1024, mode: str = "auto"):
        cfg = sae.cfg
        if cfg.jumprelu_sparsity_loss_mode != "step" or cfg.pre_act_loss_coefficient is not None:
            raise NotImplementedError("the native JumpReLU step implements the 'step' L0 loss without pre-act loss")
        super().__init__(sae, lr=lr, beta1=beta1, beta2=beta2, eps=eps, max_grad_norm=max_grad_norm,
                         h_buffer_bytes=h_buffer_bytes)
        self.k = int(min(cap, self.N))
        self.bandwidth = float(cfg.jumprelu_bandwidth)
        self.l0_coef = float(cfg.l0_coefficient)
        dev = self.device
        self.p_lthr = sae.log_threshold.detach().to(device=dev, dtype=torch.float32).clone()
        sae.log_threshold = nn.Parameter(self.p_lthr, requires_grad=False)
        self.m_lthr, self.v_lthr = torch.zeros_like(self.p_lthr), torch.zeros_like(self.p_lthr)
        self.g_thr = torch.zeros_like(self.p_lthr)
        self.truncated = torch.zeros(1, dtype=torch.int32, device=dev)
        self.last_l0 = torch.zeros((), device=dev)
        if mode not in ("auto", "dense", "sparse"):
            raise ValueError("mode must be 'auto', 'dense' or 'sparse'")
        self.policy = mode
        self.mode = "sparse" if mode == "sparse" else "dense"
        self.dense_steps = self.sparse_steps = self.fallbacks = 0
        self._hold = 0
        self._dense_colptr = torch.arange(self.N + 1, dtype=torch.int64, device=dev)  # every row has a gradient
        self._nnz = torch.zeros(1, dtype=torch.int64, device=dev)
        self._fire_f = torch.zeros(self.N, dtype=torch.float32, device=dev)

    def set_coefficients(self, coefficients: dict[str, float]) -> None:
        if "l0" in coefficients:
            self.l0_coef = float(coefficients["l0"])

    def optimizer_state(self) -> dict[str, dict[str, Any]]:
        st = super().optimizer_state()
        st["log_threshold"] = {"step": torch.tensor(float(self.step_count)), "exp_avg": self.m_lthr,
                               "exp_avg_sq": self.v_lthr}
        return st

    @torch.no_grad()
    def load_optimizer_state(self, state: dict[str, dict[str, Any]]) -> None:
        super().load_optimizer_state(state)
        if "log_threshold" in state:
            self.m_lthr.copy_(state["log_threshold"]["exp_avg"].to(self.m_lthr))
            self.v_lthr.copy_(state["log_threshold"]["exp_avg_sq"].to(self.v_lthr))

    @torch.no_grad()
    def step(self, x: torch.Tensor, lr: float | None = None, dead_mask: torch.Tensor | None = None,
             want_sae_out: bool = False, act_freq: torch.Tensor | None = None,
             since_fired: torch.Tensor | None = None, run_aux: bool = False, update: bool = True) -> EngineStepResult:
        kw = dict(lr=lr, want_sae_out=want_sae_out, act_freq=act_freq, since_fired=since_fired, update=update)
        if self.mode == "sparse":
            res = self._sparse_step(x, **kw)
            if res is not None:
                self.sparse_steps += 1
                return res
            # a row exceeded the candidate cap: this step runs dense, and so do the next ones
            self.fallbacks += 1
            self.mode = "dense"
            self._hold = self.DENSE_HOLD
            warnings.warn(f"JumpReLU native step: a row has more than {self.k} entries above threshold - "
                          "bandwidth/2; running the dense form", RuntimeWarning, stacklevel=2)
        res = self._dense_step(x, **kw)
        self.dense_steps += 1
        if self.policy == "auto":
            self._hold = max(0, self._hold - 1)
            if self._hold == 0 and self.dense_steps % self.SPARSE_CHECK_EVERY == 0 and float(self.last_l0) < self.k / 8:
                self.mode = "sparse"
        return res

    @torch.no_grad()
    def _dense_step(self, x: torch.Tensor, lr: float | None, want_sae_out: bool, act_freq: torch.Tensor | None,
                    since_fired: torch.Tensor | None, update: bool) -> EngineStepResult:
        from saelens_b200 import ops

        nat, dev = self.native, self.device
        B = x.shape[0]
        D, N = self.D, self.N
        st = self.status
        xb = x if (x.dtype == torch.bfloat16 and x.is_contiguous()) else x.to(torch.bfloat16).contiguous()
        thr = self.p_lthr.exp().contiguous()
        self._mark("start")
        H = torch.empty(B, N, dtype=torch.bfloat16, device=dev)
        F = torch.empty(B, N, dtype=torch.bfloat16, device=dev)
        self._fire_f.zero_()
        self._nnz.zero_()
        ops.gemm_dense(xb, self.w_enc, out=F, out2=H, bias=self.bias_eff, thr=thr, colcnt=self._fire_f,
                       nnz=self._nnz, status=st)
        self._mark("encoder_gemm")
        sae_out = torch.empty(B, D, dtype=torch.bfloat16, device=dev) if want_sae_out else None
        mse_sum = torch.zeros(1, dtype=torch.float32, device=dev)
        bsum = torch.zeros(D, dtype=torch.float32, device=dev)
        dxhat = ops.gemm_dense(F, self.w_dec, b_mn=True, bias=self.p_bdec, target=xb, res_coef=2.0 / B,
                               loss=mse_sum, colsum=bsum, out2=sae_out, status=st)
        mse = mse_sum[0] / B
        l0 = self._nnz[0].to(torch.float32) / B
        l0_loss = self.l0_coef * l0
        self._mark("decode_mse")
        self.sumsq.zero_()
        ops.gemm_dense(F, dxhat, a_mn=True, b_mn=True, out=self.g_dec, sumsq=self.sumsq, status=st)
        self.g_thr.zero_()
        self.g_benc.zero_()
        dH = F  # F is not read again: dL/dH takes its buffer
        ops.gemm_dense(dxhat, self.w_dec, out=dH, hin=H, thr=thr, bandwidth=self.bandwidth,
                       l0c=self.l0_coef / (B * self.bandwidth), gthr=self.g_thr, colsum=self.g_benc, status=st)
        del H
        r1 = dict(r1_row=self.g_benc, r1_col=self.p_bdec) if self.apply_b_dec else {}
        ops.gemm_dense(dH, xb, a_mn=True, b_mn=True, out=self.g_enc, sumsq=self.sumsq, status=st, **r1)
        del dH, F
        self.launches += 5
        fired = self._fire_f
        self.fire_counts.copy_(fired.to(torch.int32))
        if act_freq is not None:
            act_freq.add_(fired)
        if since_fired is not None:
            since_fired.add_(1.0).mul_((fired == 0).to(since_fired.dtype))
        g_lthr = self.g_thr * thr
        self.sumsq += self.g_benc.square().sum() + g_lthr.square().sum()
        bterm = (self.g_benc.to(torch.bfloat16)[None] @ self.w_enc).float()[0] if self.apply_b_dec else None
        self._mark("gradients")
        if update:
            self._adam(lr, bsum, bterm, g_lthr, self._dense_colptr)
            self._mark("adam")
        self.last_l0 = l0
        self.last_loss = mse + l0_loss
        return EngineStepResult(loss=mse + l0_loss, mse_loss=mse, aux_loss=l0_loss, sae_out=sae_out,
                                topk_vals=None, topk_idx=None, fire_counts=self.fire_counts, l0=l0)

    def _adam(self, lr: float | None, bsum: torch.Tensor, bterm: torch.Tensor | None, g_lthr: torch.Tensor,
              colptr: torch.Tensor) -> None:
        nat = self.native
        self.step_count += 1
        cur_lr = self.lr if lr is None else lr
        nat.adam_bdec(bsum, bterm if self.apply_b_dec else None, self.g_bdec, self.sumsq, self.clip,
                      self.p_bdec, self.m_bdec, self.v_bdec, cur_lr, self.beta1, self.beta2, self.eps,
                      self.step_count, self.max_grad_norm, True)
        nat.adam_rows(self.p_dec, self.m_dec, self.v_dec, self.p_enc, self.m_enc, self.v_enc, self.w_dec,
                      self.w_enc, self.g_dec, self.g_enc, self.p_benc, self.m_benc, self.v_benc, self.g_benc,
                      colptr, self.clip, self.p_bdec if self.apply_b_dec else None, self.scale,
                      self.inv_scale, self.bias_eff, cur_lr, self.beta1, self.beta2, self.eps,
                      self.step_count, True)
        # Adam on log_threshold (same formula as the row kernel; clip factor from the device)
        g = g_lthr * self.clip
        b1, b2 = self.beta1, self.beta2
        self.m_lthr.mul_(b1).add_(g, alpha=1 - b1)
        self.v_lthr.mul_(b2).addcmul_(g, g, value=1 - b2)
        bc1, bc2 = 1 - b1 ** self.step_count, 1 - b2 ** self.step_count
        self.p_lthr.addcdiv_(self.m_lthr, self.v_lthr.sqrt() / math.sqrt(bc2) + self.eps, value=-cur_lr / bc1)
        self.launches += 2

    @torch.no_grad()
    def _sparse_step(self, x: torch.Tensor, lr: float | None, want_sae_out: bool, act_freq: torch.Tensor | None,
                     since_fired: torch.Tensor | None, update: bool) -> EngineStepResult | None:
        nat, dev = self.native, self.device
        B = x.shape[0]
        D, N, cap = self.D, self.N, self.k
        xb = x if (x.dtype == torch.bfloat16 and x.is_contiguous()) else x.to(torch.bfloat16).contiguous()
        thr = self.p_lthr.exp()
        lo = (thr - self.bandwidth / 2).contiguous()
        lo_cmin = lo.view(N // 32, 32).amin(1).contiguous()
        self._mark("start")
        R = self._row_chunk(B)
        H = torch.empty(min(R, B), N, dtype=torch.bfloat16, device=dev)
        cm = torch.empty(min(R, B), N // 32, dtype=torch.bfloat16, device=dev)
        pre = torch.empty(B, cap, dtype=torch.float32, device=dev)
        idx = torch.empty(B, cap, dtype=torch.int32, device=dev)
        counts = torch.empty(B, dtype=torch.int32, device=dev)
        for r0 in range(0, B, R):
            r1 = min(B, r0 + R)
            h, c = H[: r1 - r0], cm[: r1 - r0]
            nat.gemm_tn_bf16(xb[r0:r1], self.w_enc, self.bias_eff, None, False, h, c, self.status.tensor, 0)
            nat.threshold_select(h, c, lo, lo_cmin, pre[r0:r1], idx[r0:r1], counts[r0:r1], self.truncated)
            self.launches += 2
        del H, cm
        self._mark("encoder_gemm_select")
        if int(self.truncated.item()) > 0:  # host sync: a row does not fit the candidate cap
            self.truncated.zero_()
            return None
        valid = idx >= 0
        safe = idx.clamp(min=0).long()
        active = valid & (pre > thr[safe])
        acts = torch.where(active, pre, torch.zeros_like(pre))
        l0 = active.sum(1).float().mean()
        # decode + MSE + dL/dx_hat over the active entries
        sae_out = torch.empty(B, D, dtype=torch.bfloat16, device=dev) if want_sae_out else None
        dxhat = torch.empty(B, D, dtype=torch.bfloat16, device=dev)
        loss_row = torch.empty(B, dtype=torch.float32, device=dev)
        bsum = torch.zeros(D, dtype=torch.float32, device=dev)
        nat.decode_mse(acts, idx, True, None, self.w_dec, self.p_bdec, xb, sae_out, None, dxhat, None, 2.0 / B,
                       loss_row, bsum)
        mse = loss_row.sum() / B
        l0_loss = self.l0_coef * l0
        self.launches += 1
        self._mark("decode_mse")
        # pair lists over every candidate (active or in the threshold window)
        marker = valid.to(torch.float32)
        self.counts.zero_()
        self.cursor.zero_()
        nat.csc_count(marker, idx, None, None, self.counts, None)
        torch.cumsum(self.counts, 0, out=self.colptr[1:])
        pairs = torch.empty(B * cap, dtype=torch.int64, device=dev)
        nat.csc_fill(marker, idx, None, None, self.colptr, self.cursor, pairs)
        fired = torch.zeros(N, dtype=torch.float32, device=dev)
        fired.index_add_(0, safe[active], torch.ones_like(pre[active]))
        self.fire_counts.copy_(fired.to(torch.int32))
        self._mark("csc_build")
        self.sumsq.zero_()
        self.g_thr.zero_()
        bterm = torch.zeros(D, dtype=torch.float32, device=dev)
        nat.latent_grad(self.colptr, pairs, marker, None, None, dxhat, None, xb,
                        self.p_bdec if self.apply_b_dec else None, self.w_dec, self.w_enc, self.g_dec, self.g_enc,
                        self.g_benc, bterm if self.apply_b_dec else None, self.sumsq, self.fire_counts, act_freq,
                        since_fired, idx, None, 0, -1, False, thr.contiguous(), pre, self.bandwidth,
                        self.l0_coef / (B * self.bandwidth), self.g_thr)
        self.launches += 3
        g_lthr = self.g_thr * thr
        self.sumsq += g_lthr.square().sum()
        self._mark("latent_grad")
        if update:
            self._adam(lr, bsum, bterm, g_lthr, self.colptr)
            self._mark("adam")
        self.last_l0 = l0
        self.last_loss = mse + l0_loss
        return EngineStepResult(loss=mse + l0_loss, mse_loss=mse, aux_loss=l0_loss, sae_out=sae_out,
                                topk_vals=acts, topk_idx=torch.where(active, idx, torch.full_like(idx, -1)),
                                fire_counts=self.fire_counts)


def jumprelu_engine_supported(sae: Any) -> bool:
    from saelens_b200 import ops
    from saelens_b200.models.jumprelu import JumpReLUTrainingSAE

    if type(sae) is not JumpReLUTrainingSAE or not sae.W_dec.is_cuda or not ops.available():
        return False
    N, D = sae.W_dec.shape
    return (D % 64 == 0 and N % 256 == 0 and sae.cfg.jumprelu_sparsity_loss_mode == "step"
            and sae.cfg.pre_act_loss_coefficient is None
            and sae.cfg.normalize_activations in ("none", "expected_average_only_in"))
