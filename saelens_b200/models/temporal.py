"""TemporalSAE (inference): causal attention over the sequence predicts part of each code, the
rest (the novel part) goes through a sparse SAE (sae_lens/saes/temporal_sae.py, arXiv:2511.01836).
Attention runs on torch SDPA with `is_causal=True`."""

from __future__ import annotations

import logging
import math
from dataclasses import dataclass
from typing import Literal

import torch
import torch.nn.functional as F
from torch import nn

from saelens_b200.models.sae import SAE, SAEConfig

logger = logging.getLogger("saelens_b200")


def get_attention(query: torch.Tensor, key: torch.Tensor) -> torch.Tensor:
    """Explicit causal attention weights (for inspection; the forward uses SDPA)."""
    L, S = query.size(-2), key.size(-2)
    w = query @ key.transpose(-2, -1) / math.sqrt(query.size(-1))
    mask = torch.ones(L, S, dtype=torch.bool, device=query.device).tril()
    w = w.masked_fill(~mask, float("-inf"))
    return torch.softmax(w, dim=-1)


def _row_normalised_(lin: nn.Linear, scale: float) -> None:
    with torch.no_grad():
        w = lin.weight
        w.copy_(scale * w / (1e-6 + torch.linalg.norm(w, dim=1, keepdim=True)))


class ManualAttention(nn.Module):
    def __init__(self, dimin: int, n_heads: int = 4, bottleneck_factor: int = 64, bias_k: bool = True,
                 bias_q: bool = True, bias_v: bool = True, bias_o: bool = True):
        super().__init__()
        if dimin % (bottleneck_factor * n_heads) != 0:
            raise ValueError("dimin must be divisible by bottleneck_factor * n_heads")
        self.n_heads = n_heads
        self.n_embds = dimin // bottleneck_factor
        self.dimin = dimin
        self.k_ctx = nn.Linear(dimin, self.n_embds, bias=bias_k)
        self.q_target = nn.Linear(dimin, self.n_embds, bias=bias_q)
        self.v_ctx = nn.Linear(dimin, dimin, bias=bias_v)
        self.c_proj = nn.Linear(dimin, dimin, bias=bias_o)
        _row_normalised_(self.k_ctx, 1 / math.sqrt(self.n_embds // n_heads))
        _row_normalised_(self.q_target, 1 / math.sqrt(self.n_embds // n_heads))
        _row_normalised_(self.v_ctx, 1 / math.sqrt(dimin // n_heads))
        _row_normalised_(self.c_proj, 1 / math.sqrt(dimin))

    def forward(self, x_ctx: torch.Tensor, x_target: torch.Tensor,
                get_attn_map: bool = False) -> tuple[torch.Tensor, torch.Tensor | None]:
        B, T, _ = x_ctx.shape
        h = self.n_heads
        k = self.k_ctx(x_ctx).view(B, T, h, -1).transpose(1, 2)
        q = self.q_target(x_target).view(B, T, h, -1).transpose(1, 2)
        v = self.v_ctx(x_ctx).view(B, T, h, -1).transpose(1, 2)
        amap = get_attention(q, k) if get_attn_map else None
        o = F.scaled_dot_product_attention(q, k, v, attn_mask=None, dropout_p=0.0, is_causal=True)
        return self.c_proj(o.transpose(1, 2).reshape(B, T, self.dimin)), amap


@dataclass
class TemporalSAEConfig(SAEConfig):
    n_heads: int = 8
    n_attn_layers: int = 1
    bottleneck_factor: int = 64
    sae_diff_type: Literal["relu", "topk"] = "topk"
    kval_topk: int | None = None
    tied_weights: bool = True
    activation_normalization_factor: float = 1.0

    def __post_init__(self) -> None:
        if self.normalize_activations not in (
            "none", "expected_average_only_in", "constant_norm_rescale", "constant_scalar_rescale",
            "layer_norm",
        ):
            raise ValueError(
                "normalize_activations must be none, expected_average_only_in, layer_norm, "
                f"constant_norm_rescale, or constant_scalar_rescale. Got {self.normalize_activations}"
            )

    @classmethod
    def architecture(cls) -> str:
        return "temporal"


class TemporalSAE(SAE[TemporalSAEConfig]):
    def __init__(self, cfg: TemporalSAEConfig, use_error_term: bool = False):
        super().__init__(cfg, use_error_term)
        self.attn_layers = nn.ModuleList([
            ManualAttention(cfg.d_sae, n_heads=cfg.n_heads, bottleneck_factor=cfg.bottleneck_factor)
            .to(device=self.device, dtype=self.dtype)
            for _ in range(cfg.n_attn_layers)
        ])
        self.eps = 1e-6
        self.lam = 1 / (4 * cfg.d_in)
        self.setup()

    def _setup_activation_normalization(self) -> None:
        if self.cfg.normalize_activations == "constant_scalar_rescale":
            f = self.cfg.activation_normalization_factor
            self.run_time_activation_norm_fn_in = lambda x: x * f
            self.run_time_activation_norm_fn_out = lambda x: x / f
        else:
            super()._setup_activation_normalization()

    def initialize_weights(self) -> None:
        c = self.cfg
        self.W_dec = nn.Parameter(torch.randn(c.d_sae, c.d_in, dtype=self.dtype, device=self.device))
        self.b_dec = nn.Parameter(torch.zeros(c.d_in, dtype=self.dtype, device=self.device))
        if not c.tied_weights:
            self.W_enc = nn.Parameter(torch.randn(c.d_in, c.d_sae, dtype=self.dtype, device=self.device))

    def _enc_matrix(self) -> torch.Tensor:
        return self.W_dec.T if self.cfg.tied_weights else self.W_enc

    def encode_with_predictions(self, x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        x = self.process_sae_in(x)
        B, L, _ = x.shape
        W_enc = self._enc_matrix()
        resid = x
        z_pred = torch.zeros(B, L, self.cfg.d_sae, device=x.device, dtype=x.dtype)
        for layer in self.attn_layers:
            z_in = F.relu((resid * self.lam) @ W_enc)
            z_ctx = torch.cat((torch.zeros_like(z_in[:, :1]), z_in[:, :-1].clone()), dim=1)
            zp, _ = layer(z_ctx, z_in)
            zp = F.relu(zp)
            dz = zp @ self.W_dec
            nrm = dz.norm(dim=-1, keepdim=True) + self.eps
            proj = (dz * resid).sum(dim=-1, keepdim=True) / nrm.pow(2)
            z_pred = z_pred + zp * proj
            resid = resid - proj * dz
        z_novel = F.relu((resid * self.lam) @ W_enc)
        if self.cfg.sae_diff_type == "topk" and self.cfg.kval_topk is not None:
            _, idx = torch.topk(z_novel, self.cfg.kval_topk, dim=-1)
            z_novel = z_novel * torch.zeros_like(z_novel).scatter_(-1, idx, 1)
        return z_novel, z_pred

    def encode(self, x: torch.Tensor) -> torch.Tensor:
        return self.encode_with_predictions(x)[0]

    def decode(self, feature_acts: torch.Tensor) -> torch.Tensor:
        out = self.hook_sae_recons(feature_acts @ self.W_dec + self.b_dec)
        out = self.run_time_activation_norm_fn_out(out)
        logger.warning("TemporalSAE.decode only decodes the novel codes; forward() adds the predicted part.")
        return out

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        zn, zp = self.encode_with_predictions(x)
        out = (zn + zp) @ self.W_dec + self.b_dec
        return self.hook_sae_output(self.run_time_activation_norm_fn_out(out))

    def fold_W_dec_norm(self) -> None:
        raise NotImplementedError("Folding W_dec_norm is not supported for TemporalSAE")

    @torch.no_grad()
    def fold_activation_norm_scaling_factor(self, scaling_factor: float) -> None:
        raise NotImplementedError("Folding activation norm scaling factor is not supported for TemporalSAE")
