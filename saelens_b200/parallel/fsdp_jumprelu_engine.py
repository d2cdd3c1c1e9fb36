"""Sharded data-parallel (FSDP-style) JumpReLU training step on several B200s.

Layout and protocol as `FSDPTopKEngine`: rank r of S owns latents [r*n, (r+1)*n) with their fp32
masters, Adam moments, b_enc and log_threshold; b_dec is replicated; the bf16 W_enc / W_dec live in
full [d_sae, d_in] buffers in every rank's symmetric slab.  Reference semantics: torch FSDP
FULL_SHARD around the JumpReLU training forward (sae_lens/llm_sae_training_runner.py:449-463,
sae_lens/saes/jumprelu_sae.py:19-85, 241-312).  The step is the dense form of the single-GPU
JumpReLU step (`JumpReLUEngine`), which holds at any sparsity:

  1. encoder GEMM with the parameter all-gather fused in and the JumpReLU epilogue
     (`gemm_fsdp_dense_bf16`): H (pre-activations), F = H 1[H > theta], firing counts, L0 count;
  2. after the W_dec flags: x_hat = F W_dec + b_dec with the MSE, dL/dx_hat and its column sums;
  3. gW_dec = F^T dL/dx_hat with the reduce-scatter fused into the epilogue: every output row is
     stored over NVLink into the landing slot of the rank that owns its latent;
  4. dL/dH (JumpReLU backward, rectangle-window threshold gradient, b_enc column sums);
  5. gW_enc = dL/dH^T x - gb_enc (x) b_dec, reduce-scattered the same way; then a release flag
     per (source, owner);
  6. the owner sums its S slots (1/S) with the squared norm; one P2P all-reduce averages
     [gb_enc | b_dec terms | mse | L0 | norm part | threshold gradient], one sums the firing counts;
  7. clip + Adam on the shard (rows, b_enc, log_threshold), then the per-latent vectors (folded
     bias, ||W_dec||, threshold) are regathered for the next step's epilogues.
The buffer-reuse argument of `FSDPTopKEngine` holds unchanged: the landing slots and weight
buffers are written and read in the same order.
"""

from __future__ import annotations

import math
from typing import Any

import torch
import torch.distributed as dist
from torch import nn

from saelens_b200.parallel.fsdp_engine import FSDPTopKEngine
from saelens_b200.training.engine import EngineStepResult


class FSDPJumpReLUEngine(FSDPTopKEngine):
    aux_loss_name = "l0_loss"
    N_VECS = 4  # + threshold

    def _extra_small(self) -> int:
        return int(self.N_full)  # threshold gradient of every latent

    def __init__(self, sae: Any, lr: float, group: dist.ProcessGroup | None, beta1: float = 0.9,
                 beta2: float = 0.999, eps: float = 1e-8, max_grad_norm: float = 1.0):
        cfg = sae.cfg
        if cfg.jumprelu_sparsity_loss_mode != "step" or cfg.pre_act_loss_coefficient is not None:
            raise NotImplementedError("the native JumpReLU step implements the 'step' L0 loss without pre-act loss")
        rank, world = dist.get_rank(group), dist.get_world_size(group)
        N = sae.W_dec.shape[0]
        n = N // world
        lthr_full = sae.log_threshold.detach()
        # the shard's log_threshold (fp32) is set before the parent gathers the per-latent vectors
        self.p_lthr = lthr_full[rank * n : (rank + 1) * n].to(device=sae.W_dec.device, dtype=torch.float32).clone()
        sae.log_threshold = nn.Parameter(self.p_lthr, requires_grad=False)
        self.bandwidth = float(cfg.jumprelu_bandwidth)
        self.l0_coef = float(cfg.l0_coefficient)
        super().__init__(sae, lr=lr, group=group, beta1=beta1, beta2=beta2, eps=eps, max_grad_norm=max_grad_norm)
        self.m_lthr, self.v_lthr = torch.zeros_like(self.p_lthr), torch.zeros_like(self.p_lthr)
        self.last_l0 = torch.zeros((), device=self.device)

    def k_request(self) -> int:
        return 1  # no per-row selection: the dense form keeps no candidate lists

    def _vector_parts(self) -> list[torch.Tensor]:
        return [self.bias_eff, self.scale, self.inv_scale, self.p_lthr.exp()]

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
             since_fired: torch.Tensor | None = None, run_aux: bool = False,
             update: bool = True) -> EngineStepResult:
        from saelens_b200 import ops

        nat, dev = self.native, self.device
        S, r, n, D, NF = self.size, self.rank, self.N, self.D, self.N_full
        st, tk, bases = self.status, self._ticket, self.heap.bases
        B = x.shape[0]
        xb = x if (x.dtype == torch.bfloat16 and x.is_contiguous()) else x.to(torch.bfloat16).contiguous()
        ep = self._epoch("step")
        thr_full = self.vec_full[3]
        self._mark("start")

        # 1. all-gather fused encoder GEMM with the JumpReLU epilogue
        H = torch.empty(B, NF, dtype=torch.bfloat16, device=dev)
        F = torch.empty(B, NF, dtype=torch.bfloat16, device=dev)
        fire = torch.zeros(NF, dtype=torch.float32, device=dev)
        nnz = torch.zeros(1, dtype=torch.int64, device=dev)
        nat.gemm_fsdp_dense_bf16(xb, self.w_enc, bases, r, self.wenc_buf.offset, self.wenc_flags.offset, True, ep,
                                 self.w_dec, self.wdec_buf.offset, self.wdec_flags.offset, F, H, self.bias_full,
                                 thr_full, fire, nnz, st.tensor, tk)
        self._mark("fsdp_encoder_gemm")

        # 2. decode + MSE + dL/dx_hat with the gathered W_dec
        nat.p2p_wait_flags(self.wdec_flags_local, ep, st.tensor)
        small = torch.zeros(self._small_n, dtype=torch.float32, device=dev)
        gb, bsum, bterm = small[:NF], small[NF : NF + D], small[NF + D : NF + 2 * D]
        o = NF + 2 * D
        gthr = small[o + 3 :]
        mse_sum = torch.zeros(1, dtype=torch.float32, device=dev)
        sae_out = torch.empty(B, D, dtype=torch.bfloat16, device=dev) if want_sae_out else None
        dxhat = ops.gemm_dense(F, self.wdec_full, b_mn=True, bias=self.p_bdec, target=xb, res_coef=2.0 / B,
                               loss=mse_sum, colsum=bsum, out2=sae_out, status=st)
        self._mark("decode_mse")

        # 3-5. gradients; the weight-gradient rows go straight to their owners' landing slots
        ops.gemm_dense(F, dxhat, a_mn=True, b_mn=True, want_out=False, status=st, rs_bases=bases, rs_rank=r,
                       rs_off=self.land_dec.offset, rs_n=n)
        dH = F
        ops.gemm_dense(dxhat, self.wdec_full, out=dH, hin=H, thr=thr_full, bandwidth=self.bandwidth,
                       l0c=self.l0_coef / (B * self.bandwidth), gthr=gthr, colsum=gb, status=st)
        del H
        r1 = dict(r1_row=gb, r1_col=self.p_bdec) if self.apply_b_dec else {}
        ops.gemm_dense(dH, xb, a_mn=True, b_mn=True, want_out=False, status=st, rs_bases=bases, rs_rank=r,
                       rs_off=self.land_enc.offset, rs_n=n, **r1)
        del dH, F
        if self.apply_b_dec:
            bterm.copy_((gb.to(torch.bfloat16)[None] @ self.wenc_full).float()[0])
        nat.p2p_signal(bases, r, self.gflags.offset, r, self._all_mask, ep)
        self.launches += 6
        self._mark("gradients_reduce_scatter")

        # 6. owner: sum the slots; average the small vector; sum the firing counts
        nat.p2p_wait_flags(self.gflags_local, ep, st.tensor)
        part = torch.zeros(1, dtype=torch.float32, device=dev)
        nat.p2p_slot_reduce(self.land_dec_local, 1.0 / S, self.g_dec, part)
        nat.p2p_slot_reduce(self.land_enc_local, 1.0 / S, self.g_enc, part)
        small[o] = mse_sum[0] / B
        small[o + 1] = nnz[0].to(torch.float32) / B
        small[o + 2] = part[0] * S  # summed (not averaged) by the 1/S all-reduce
        self.launches += 3
        red = self._ar(small, self.small, "small", 1.0 / S)
        fired = self._ar(fire, self.fire, "fire", 1.0)
        self._mark("grad_reduce")
        if act_freq is not None:
            act_freq += fired
        if since_fired is not None:
            since_fired.copy_(torch.where(fired > 0, torch.zeros_like(since_fired), since_fired + 1))
        fire_counts = fired.round().to(torch.int32)
        gb_all, gthr_all = red[:NF], red[o + 3 :]
        g_lthr_all = gthr_all * thr_full
        sumsq = (red[o + 2] + gb_all.square().sum() + g_lthr_all.square().sum()).reshape(1)
        self.sumsq = sumsq
        mse, l0 = red[o], red[o + 1]
        l0_loss = self.l0_coef * l0

        # 7. clip + Adam on the shard; per-latent vectors regathered
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
            g = g_lthr_all[r * n : (r + 1) * n] * self.clip
            b1, b2 = self.beta1, self.beta2
            self.m_lthr.mul_(b1).add_(g, alpha=1 - b1)
            self.v_lthr.mul_(b2).addcmul_(g, g, value=1 - b2)
            bc1, bc2 = 1 - b1 ** self.step_count, 1 - b2 ** self.step_count
            self.p_lthr.addcdiv_(self.m_lthr, self.v_lthr.sqrt() / math.sqrt(bc2) + self.eps, value=-cur_lr / bc1)
            self.launches += 2
            self._gather_vectors()
            self._mark("adam")
        self.last_l0 = l0
        self.last_loss = mse + l0_loss
        return EngineStepResult(loss=mse + l0_loss, mse_loss=mse, aux_loss=l0_loss, sae_out=sae_out,
                                topk_vals=None, topk_idx=None, fire_counts=fire_counts, l0=l0)

    def full_weights(self) -> dict[str, torch.Tensor]:
        out = super().full_weights()
        parts = [torch.empty_like(self.p_lthr) for _ in range(self.size)]
        dist.all_gather(parts, self.p_lthr.contiguous(), group=self.group)
        out["log_threshold"] = torch.cat(parts)
        return out


def fsdp_jumprelu_supported(sae: Any, world: int) -> bool:
    from saelens_b200.training.jumprelu_engine import jumprelu_engine_supported

    return jumprelu_engine_supported(sae) and sae.W_dec.shape[0] % (256 * world) == 0


__all__ = ["FSDPJumpReLUEngine", "fsdp_jumprelu_supported"]
