"""Native Matryoshka BatchTopK training step (sae_lens/saes/matryoshka_batchtopk_sae.py:86-150).

The loss adds, to the BatchTopK loss of the full dictionary, the MSE of every inner prefix
reconstruction: with widths w_1 < ... < w_L = d_sae, x_hat_l = b_dec + sum over the selected
latents j < w_l of a_j W_dec_j, and loss = sum_l MSE(x_hat_l, x) + aux.  A latent j in level l
(w_{l-1} <= j < w_l) appears in every reconstruction of level >= l, so its gradients use
G_l = sum_{i >= l} dL/dx_hat_i, the suffix sum of the levels' dL/dx_hat:

  1. encoder GEMM, row top-k and the batch-wide selection as in `FusedTopKEngine`;
  2. one sparse partial decode per level (the level's selected latents only, fp32), whose running
     sums are the nested reconstructions; their MSEs and dL/dx_hat, and the suffix sums G_l;
  3. the dead-latent aux loss against the full reconstruction (as the base engine);
  4. the CSC pair lists once, then one latent-gradient launch per level over that level's latent
     range with G_l as the reconstruction gradient (the kernels take a latent range);
  5. clip + row-fused Adam as the base engine.
"""

from __future__ import annotations

from typing import Any

import torch

from saelens_b200.training.engine import EngineStepResult, FusedTopKEngine, _StepState


class MatryoshkaEngine(FusedTopKEngine):
    def __init__(self, sae: Any, lr: float, **kw: Any):
        super().__init__(sae, lr=lr, **kw)
        widths = [int(w) for w in sae.cfg.matryoshka_widths]
        if not widths or widths[-1] != self.N or any(a >= b for a, b in zip(widths[:-1], widths[1:])):
            raise ValueError("matryoshka_widths must be strictly increasing and end at d_sae")
        self.widths = widths
        self._bounds = torch.tensor(widths, dtype=torch.int64, device=self.device)

    @torch.no_grad()
    def step(self, x: torch.Tensor, lr: float | None = None, dead_mask: torch.Tensor | None = None,
             want_sae_out: bool = False, act_freq: torch.Tensor | None = None,
             since_fired: torch.Tensor | None = None, run_aux: bool = False,
             update: bool = True) -> EngineStepResult:
        nat, dev, D = self.native, self.device, self.D
        fw = self._encode_select(x, dead_mask, run_aux)
        B, xb, vals, idx, aux_on = fw["B"], fw["xb"], fw["vals"], fw["idx"], fw["aux_on"]
        inv = self.inv_scale if self.rescale else None
        # 2. nested reconstructions: level l holds the selected latents in [w_{l-1}, w_l)
        level = torch.where(idx >= 0, torch.bucketize(idx.clamp(min=0).to(torch.int64), self._bounds, right=True),
                            torch.full_like(idx, -1, dtype=torch.int64))
        xf = xb.float()
        cum = self.p_bdec[None].expand(B, D).clone()
        dxs: list[torch.Tensor] = []
        mses: list[torch.Tensor] = []
        part = torch.empty(B, D, dtype=torch.float32, device=dev)
        for li in range(len(self.widths)):
            v_l = torch.where(level == li, vals, torch.zeros_like(vals)).contiguous()
            part.zero_()
            nat.decode_partial(v_l, idx, True, inv, self.w_dec, part)
            cum += part
            recon = cum.to(torch.bfloat16).float()  # the model's bf16 reconstruction
            diff = recon - xf
            mses.append(diff.square().sum(-1).mean())
            dxs.append(diff * (2.0 / B))
        self.launches += len(self.widths)
        sae_out = cum.to(torch.bfloat16) if (want_sae_out or aux_on) else None
        resid = (xf - cum.to(torch.bfloat16).float()).to(torch.bfloat16) if aux_on else None
        # suffix sums G_l = sum_{i >= l} dL/dx_hat_i (bf16 for the gradient kernels)
        G: list[torch.Tensor] = [torch.empty(0)] * len(dxs)
        acc = torch.zeros(B, D, dtype=torch.float32, device=dev)
        for li in range(len(dxs) - 1, -1, -1):
            acc += dxs[li]
            G[li] = acc.to(torch.bfloat16)
        bsum = acc.sum(0)  # every level's dL/dx_hat reaches b_dec
        self._mark("decode_mse")
        daux, aux_loss = self._aux_decode(fw, resid)
        pairs = self._build_csc(fw)
        # 4. latent gradients level by level (latent ranges of the CSC lists)
        self.sumsq.zero_()
        bterm = torch.zeros(D, dtype=torch.float32, device=dev)
        j0 = 0
        for li, w in enumerate(self.widths):
            nat.latent_grad(self.colptr, pairs, vals, fw.get("aux_vals"), inv, G[li], daux, xb,
                            self.p_bdec if self.apply_b_dec else None, self.w_dec, self.w_enc, self.g_dec, self.g_enc,
                            self.g_benc, bterm if self.apply_b_dec else None, self.sumsq, self.fire_counts, act_freq,
                            since_fired, idx, fw.get("aux_idx"), j0, w)
            j0 = w
        self.launches += 3 * len(self.widths)
        self._mark("latent_grad")
        outer = mses[-1]
        inner = {f"inner_mse_loss_{w}": m for w, m in zip(self.widths[:-1], mses[:-1])}
        total_mse_extra = sum(mses[:-1], torch.zeros((), device=dev))
        st = _StepState(B=B, xb=xb, vals=vals, idx=idx, aux_on=aux_on, aux_vals=fw.get("aux_vals"),
                        aux_idx=fw.get("aux_idx"), dxhat=G[0], daux=daux, bsum=bsum, pairs=pairs, mse=outer,
                        aux_loss=aux_loss, sae_out=sae_out, act_freq=act_freq, since_fired=since_fired, lr=lr,
                        update=update)
        if update:
            self._update(st, bterm)
        self.last_loss = outer + total_mse_extra + aux_loss
        return EngineStepResult(loss=self.last_loss, mse_loss=outer, aux_loss=aux_loss, sae_out=sae_out,
                                topk_vals=vals, topk_idx=idx, fire_counts=self.fire_counts, extra_losses=inner)


def matryoshka_engine_supported(sae: Any) -> bool:
    from saelens_b200 import ops
    from saelens_b200.models.batchtopk import MatryoshkaBatchTopKTrainingSAE

    if type(sae) is not MatryoshkaBatchTopKTrainingSAE or not sae.W_dec.is_cuda or not ops.available():
        return False
    N, D = sae.W_dec.shape
    return (D % 64 == 0 and N % 256 == 0 and not sae.cfg.use_matryoshka_aux_loss
            and sae.cfg.normalize_activations in ("none", "expected_average_only_in"))


__all__ = ["MatryoshkaEngine", "matryoshka_engine_supported"]
