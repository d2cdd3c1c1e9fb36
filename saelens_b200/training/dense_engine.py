"""Native training steps of the dense SAEs: Standard (ReLU + L1 weighted by ||W_dec||) and Gated.

Both run on the dense-step tcgen05 GEMM family (`ops.gemm_dense`): operands are read K-major or
MN-major in place (no transposes in memory) and the elementwise parts of the step live in the
GEMM epilogues.  fp32 masters and moments, the clip and the row-fused Adam are those of the TopK
engine (`FusedTopKEngine`).

Standard (sae_lens/saes/standard_sae.py:57-66, 137-151), loss = MSE + l1 * mean_b sum_j
F_bj ||W_dec_j||:
  1. F = relu(x W_enc^T + b_eff) with the column sums of F and the firing counts;
  2. x_hat = F W_dec + b_dec, MSE, dL/dx_hat = 2 (x_hat - x) / B and its column sums;
  3. gW_dec = F^T dL/dx_hat, plus the L1 term's (l1 / B) (sum_b F_bj) W_dec_j / ||W_dec_j||;
  4. dL/dH = (dL/dx_hat W_dec^T + (l1 / B) ||W_dec_j||) 1[F > 0] with its column sums (b_enc);
  5. gW_enc = dL/dH^T x - g_benc (x) b_dec.
Gated (sae_lens/saes/gated_sae.py:145-198): with a = (x - b_dec) W_enc^T, gate pre-activation
pi_g = a + b_gate, magnitude pre-activation pi_m = a e^r_mag + b_mag, f = 1[pi_g > 0] relu(pi_m);
loss = MSE(f W_dec + b_dec, x) + l1 * mean_b sum_j relu(pi_g)_bj ||W_dec_j|| +
MSE(relu(pi_g) W_dec + b_dec, x):
  1. one GEMM with the dual epilogue writes f and g = relu(pi_g) (and the column sums of g);
  2. two decodes (f and g paths) with their MSE, dL/dx_hat and column sums;
  3. gW_dec = [f; g]^T [dx_hat; dx_hat_aux] as one GEMM over 2B rows, plus the L1 norm term;
  4. dL/dpi_g = (dx_hat_aux W_dec^T + (l1 / B) ||W_dec||) 1[g > 0] (column sums: b_gate);
  5. dL/dpi_m = (dx_hat W_dec^T) 1[f > 0] with the column sums (b_mag) and sum_b dL/dpi_m (f - b_mag)
     (r_mag), combined in the same epilogue into dL/da = dL/dpi_m e^r + dL/dpi_g;
  6. gW_enc = dL/da^T x - (sum_b dL/da) (x) b_dec.
"""

from __future__ import annotations

import math
from typing import Any

import torch
from torch import nn

from saelens_b200.training.engine import EngineStepResult, FusedTopKEngine


class _DenseBase(FusedTopKEngine):
    aux_loss_name = "l1_loss"

    def __init__(self, sae: Any, lr: float, **kw: Any):
        super().__init__(sae, lr=lr, **kw)
        dev = self.device
        self.l1_coef = float(sae.cfg.l1_coefficient)
        self._dense_colptr = torch.arange(self.N + 1, dtype=torch.int64, device=dev)
        self._zeros_n = torch.zeros(self.N, dtype=torch.float32, device=dev)
        self._nnz = torch.zeros(1, dtype=torch.int64, device=dev)
        self._fire_f = torch.zeros(self.N, dtype=torch.float32, device=dev)
        self.last_l0 = torch.zeros((), device=dev)

    def set_coefficients(self, coefficients: dict[str, float]) -> None:
        if "l1" in coefficients:
            self.l1_coef = float(coefficients["l1"])

    def _stats(self, act_freq: torch.Tensor | None, since_fired: torch.Tensor | None) -> None:
        fired = self._fire_f
        self.fire_counts.copy_(fired.to(torch.int32))
        if act_freq is not None:
            act_freq.add_(fired)
        if since_fired is not None:
            since_fired.add_(1.0).mul_((fired == 0).to(since_fired.dtype))

    def _norm_term(self, colsum: torch.Tensor, coef: float, B: int) -> None:
        """gW_dec_j += (l1 / B) colsum_j W_dec_j / ||W_dec_j|| (the L1 penalty's pull on the norms)."""
        s = (coef / B) * colsum / self.scale.clamp(min=1e-12)
        self.g_dec.copy_((self.g_dec.float() + s[:, None] * self.w_dec.float()).to(torch.bfloat16))

    def _adam_main(self, lr: float | None, bsum: torch.Tensor, bterm: torch.Tensor | None) -> float:
        nat = self.native
        self.step_count += 1
        cur_lr = self.lr if lr is None else lr
        nat.adam_bdec(bsum, bterm if self.apply_b_dec else None, self.g_bdec, self.sumsq, self.clip,
                      self.p_bdec, self.m_bdec, self.v_bdec, cur_lr, self.beta1, self.beta2, self.eps,
                      self.step_count, self.max_grad_norm, True)
        nat.adam_rows(self.p_dec, self.m_dec, self.v_dec, self.p_enc, self.m_enc, self.v_enc, self.w_dec,
                      self.w_enc, self.g_dec, self.g_enc, self.p_benc, self.m_benc, self.v_benc, self.g_benc,
                      self._dense_colptr, self.clip, self.p_bdec if self.apply_b_dec else None, self.scale,
                      self.inv_scale, self.bias_eff, cur_lr, self.beta1, self.beta2, self.eps,
                      self.step_count, True)
        self.launches += 2
        return cur_lr

    def _adam_vec(self, p: torch.Tensor, m: torch.Tensor, v: torch.Tensor, g: torch.Tensor, lr: float) -> None:
        """Adam on a small fp32 vector with the device clip factor (same formula as the row kernel)."""
        g = g * self.clip
        b1, b2 = self.beta1, self.beta2
        m.mul_(b1).add_(g, alpha=1 - b1)
        v.mul_(b2).addcmul_(g, g, value=1 - b2)
        bc1, bc2 = 1 - b1 ** self.step_count, 1 - b2 ** self.step_count
        p.addcdiv_(m, v.sqrt() / math.sqrt(bc2) + self.eps, value=-lr / bc1)


class StandardEngine(_DenseBase):
    @torch.no_grad()
    def step(self, x: torch.Tensor, lr: float | None = None, dead_mask: torch.Tensor | None = None,
             want_sae_out: bool = False, act_freq: torch.Tensor | None = None,
             since_fired: torch.Tensor | None = None, run_aux: bool = False, update: bool = True) -> EngineStepResult:
        from saelens_b200 import ops

        dev, st = self.device, self.status
        B, D, N = x.shape[0], self.D, self.N
        xb = x if (x.dtype == torch.bfloat16 and x.is_contiguous()) else x.to(torch.bfloat16).contiguous()
        coef = self.l1_coef
        self._mark("start")
        F = torch.empty(B, N, dtype=torch.bfloat16, device=dev)
        colF = torch.zeros(N, dtype=torch.float32, device=dev)
        self._fire_f.zero_()
        self._nnz.zero_()
        ops.gemm_dense(xb, self.w_enc, out=F, bias=self.bias_eff, relu=True, colsum=colF, colcnt=self._fire_f,
                       nnz=self._nnz, status=st)
        self._mark("encoder_gemm")
        sae_out = torch.empty(B, D, dtype=torch.bfloat16, device=dev) if want_sae_out else None
        mse_sum = torch.zeros(1, dtype=torch.float32, device=dev)
        bsum = torch.zeros(D, dtype=torch.float32, device=dev)
        dxhat = ops.gemm_dense(F, self.w_dec, b_mn=True, bias=self.p_bdec, target=xb, res_coef=2.0 / B,
                               loss=mse_sum, colsum=bsum, out2=sae_out, status=st)
        mse = mse_sum[0] / B
        l1 = (coef / B) * (colF * self.scale).sum()
        self._mark("decode_mse")
        ops.gemm_dense(F, dxhat, a_mn=True, b_mn=True, out=self.g_dec, status=st)
        self._norm_term(colF, coef, B)
        self.g_benc.zero_()
        # dL/dH in F's buffer: every element is read (the ReLU mask) by the thread that overwrites it
        ops.gemm_dense(dxhat, self.w_dec, out=F, bias=(coef / B) * self.scale, hin=F, thr=self._zeros_n,
                       bandwidth=1.0, colsum=self.g_benc, status=st)
        self.sumsq.zero_()
        r1 = dict(r1_row=self.g_benc, r1_col=self.p_bdec) if self.apply_b_dec else {}
        ops.gemm_dense(F, xb, a_mn=True, b_mn=True, out=self.g_enc, sumsq=self.sumsq, status=st, **r1)
        del F
        self.sumsq += self.g_dec.float().square().sum() + self.g_benc.square().sum()
        bterm = (self.g_benc.to(torch.bfloat16)[None] @ self.w_enc).float()[0] if self.apply_b_dec else None
        self.launches += 5
        self._stats(act_freq, since_fired)
        self._mark("gradients")
        if update:
            self._adam_main(lr, bsum, bterm)
            self._mark("adam")
        l0 = self._nnz[0].to(torch.float32) / B
        self.last_l0 = l0
        self.last_loss = mse + l1
        return EngineStepResult(loss=mse + l1, mse_loss=mse, aux_loss=l1, sae_out=sae_out, topk_vals=None,
                                topk_idx=None, fire_counts=self.fire_counts, l0=l0)


class GatedEngine(_DenseBase):
    """The b_enc slot of the TopK engine's state holds b_mag (updated by the row-fused Adam with the
    b_mag gradient); b_gate and r_mag have their own fp32 masters and moments."""

    def __init__(self, sae: Any, lr: float, **kw: Any):
        object.__setattr__(sae, "b_enc", sae.b_mag)  # the parent reads the per-latent bias from b_enc
        try:
            super().__init__(sae, lr=lr, **kw)
        finally:
            sae.__dict__.pop("b_enc", None)
        dev = self.device
        self.p_bgate = sae.b_gate.detach().to(device=dev, dtype=torch.float32).clone()
        self.p_rmag = sae.r_mag.detach().to(device=dev, dtype=torch.float32).clone()
        sae.b_gate = nn.Parameter(self.p_bgate, requires_grad=False)
        sae.r_mag = nn.Parameter(self.p_rmag, requires_grad=False)
        self.m_bgate, self.v_bgate = torch.zeros_like(self.p_bgate), torch.zeros_like(self.p_bgate)
        self.m_rmag, self.v_rmag = torch.zeros_like(self.p_rmag), torch.zeros_like(self.p_rmag)
        self.g_bgate = torch.zeros_like(self.p_bgate)
        self.g_rmag = torch.zeros_like(self.p_rmag)
        self.last_aux = torch.zeros((), device=dev)

    def _alias_module(self) -> None:
        sae = self.sae
        sae.W_dec = nn.Parameter(self.p_dec, requires_grad=False)
        sae.W_enc = nn.Parameter(self.p_enc.T, requires_grad=False)
        sae.b_mag = nn.Parameter(self.p_benc, requires_grad=False)
        sae.b_dec = nn.Parameter(self.p_bdec, requires_grad=False)
        sae.dtype = torch.float32

    def optimizer_state(self) -> dict[str, dict[str, Any]]:
        st = super().optimizer_state()
        st["b_mag"] = st.pop("b_enc")
        step = torch.tensor(float(self.step_count))
        st["b_gate"] = {"step": step.clone(), "exp_avg": self.m_bgate, "exp_avg_sq": self.v_bgate}
        st["r_mag"] = {"step": step.clone(), "exp_avg": self.m_rmag, "exp_avg_sq": self.v_rmag}
        return st

    @torch.no_grad()
    def load_optimizer_state(self, state: dict[str, dict[str, Any]]) -> None:
        state = dict(state)
        if "b_mag" in state:
            state["b_enc"] = state.pop("b_mag")
        super().load_optimizer_state(state)
        for name, m, v in (("b_gate", self.m_bgate, self.v_bgate), ("r_mag", self.m_rmag, self.v_rmag)):
            if name in state:
                m.copy_(state[name]["exp_avg"].to(m))
                v.copy_(state[name]["exp_avg_sq"].to(v))

    @torch.no_grad()
    def step(self, x: torch.Tensor, lr: float | None = None, dead_mask: torch.Tensor | None = None,
             want_sae_out: bool = False, act_freq: torch.Tensor | None = None,
             since_fired: torch.Tensor | None = None, run_aux: bool = False, update: bool = True) -> EngineStepResult:
        from saelens_b200 import ops

        dev, st = self.device, self.status
        B, D, N = x.shape[0], self.D, self.N
        xb = x if (x.dtype == torch.bfloat16 and x.is_contiguous()) else x.to(torch.bfloat16).contiguous()
        coef = self.l1_coef
        e_r = self.p_rmag.exp()
        wb = (self.p_benc - self.bias_eff) if self.apply_b_dec else torch.zeros_like(self.p_benc)  # <W_enc_j, b_dec>
        gate_b = (self.p_bgate - wb).contiguous()
        mag_b = (self.p_benc - wb * e_r).contiguous()
        self._mark("start")
        FG = torch.empty(2 * B, N, dtype=torch.bfloat16, device=dev)
        F, G = FG[:B], FG[B:]
        colG = torch.zeros(N, dtype=torch.float32, device=dev)
        self._fire_f.zero_()
        self._nnz.zero_()
        ops.gemm_dense(xb, self.w_enc, out=F, out2=G, gate_bias=gate_b, mag_scale=e_r, bias=mag_b, colsum2=colG,
                       colcnt=self._fire_f, nnz=self._nnz, status=st)
        self._mark("encoder_gemm")
        sae_out = torch.empty(B, D, dtype=torch.bfloat16, device=dev) if want_sae_out else None
        DX = torch.empty(2 * B, D, dtype=torch.bfloat16, device=dev)
        mse_sum = torch.zeros(1, dtype=torch.float32, device=dev)
        aux_sum = torch.zeros(1, dtype=torch.float32, device=dev)
        bsum = torch.zeros(D, dtype=torch.float32, device=dev)
        ops.gemm_dense(F, self.w_dec, b_mn=True, out=DX[:B], bias=self.p_bdec, target=xb, res_coef=2.0 / B,
                       loss=mse_sum, colsum=bsum, out2=sae_out, status=st)
        ops.gemm_dense(G, self.w_dec, b_mn=True, out=DX[B:], bias=self.p_bdec, target=xb, res_coef=2.0 / B,
                       loss=aux_sum, colsum=bsum, status=st)
        mse, aux = mse_sum[0] / B, aux_sum[0] / B
        l1 = (coef / B) * (colG * self.scale).sum()
        self._mark("decode_mse")
        ops.gemm_dense(FG, DX, a_mn=True, b_mn=True, out=self.g_dec, status=st)
        self._norm_term(colG, coef, B)
        # dL/dpi_g in G's buffer, then dL/da (= dL/dpi_m e^r + dL/dpi_g) in F's buffer
        self.g_bgate.zero_()
        self.g_benc.zero_()
        self.g_rmag.zero_()
        ops.gemm_dense(DX[B:], self.w_dec, out=G, bias=(coef / B) * self.scale, hin=G, thr=self._zeros_n,
                       bandwidth=1.0, colsum=self.g_bgate, status=st)
        b_mag = self.p_benc.contiguous()
        ops.gemm_dense(DX[:B], self.w_dec, out=F, hin=F, thr=self._zeros_n, bandwidth=1.0, colsum=self.g_benc,
                       hsum=self.g_rmag, hoff=b_mag, addend=G, oscale=e_r, status=st)
        r1 = (self.g_benc * e_r + self.g_bgate).contiguous()  # sum_b dL/da
        self.sumsq.zero_()
        r1kw = dict(r1_row=r1, r1_col=self.p_bdec) if self.apply_b_dec else {}
        ops.gemm_dense(F, xb, a_mn=True, b_mn=True, out=self.g_enc, sumsq=self.sumsq, status=st, **r1kw)
        del FG, F, G, DX
        self.sumsq += (self.g_dec.float().square().sum() + self.g_benc.square().sum() + self.g_bgate.square().sum()
                       + self.g_rmag.square().sum())
        bterm = (r1.to(torch.bfloat16)[None] @ self.w_enc).float()[0] if self.apply_b_dec else None
        self.launches += 7
        self._stats(act_freq, since_fired)
        self._mark("gradients")
        if update:
            cur_lr = self._adam_main(lr, bsum, bterm)
            self._adam_vec(self.p_bgate, self.m_bgate, self.v_bgate, self.g_bgate, cur_lr)
            self._adam_vec(self.p_rmag, self.m_rmag, self.v_rmag, self.g_rmag, cur_lr)
            self._mark("adam")
        l0 = self._nnz[0].to(torch.float32) / B
        self.last_l0 = l0
        self.last_aux = aux
        self.last_loss = mse + l1 + aux
        return EngineStepResult(loss=mse + l1 + aux, mse_loss=mse, aux_loss=l1, sae_out=sae_out, topk_vals=None,
                                topk_idx=None, fire_counts=self.fire_counts, l0=l0,
                                extra_losses={"auxiliary_reconstruction_loss": aux})


def dense_engine_class(sae: Any) -> type | None:
    """The native engine for a Standard (L1, p = 1) or Gated training SAE on CUDA, else None."""
    from saelens_b200 import ops
    from saelens_b200.models.gated import GatedTrainingSAE
    from saelens_b200.models.standard import StandardTrainingSAE

    if not sae.W_dec.is_cuda or not ops.available():
        return None
    N, D = sae.W_dec.shape
    if D % 64 or N % 256 or sae.cfg.normalize_activations not in ("none", "expected_average_only_in"):
        return None
    if type(sae) is StandardTrainingSAE and float(sae.cfg.lp_norm) == 1.0 and isinstance(sae.activation_fn, nn.ReLU):
        return StandardEngine
    if type(sae) is GatedTrainingSAE:
        return GatedEngine
    return None


__all__ = ["StandardEngine", "GatedEngine", "dense_engine_class"]
