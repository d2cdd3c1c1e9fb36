"""Gated SAEs (sae_lens/saes/gated_sae.py): a gate path `x W_enc + b_gate > 0` and a
magnitude path `x (W_enc * exp(r_mag)) + b_mag` sharing one encoder matrix."""

from __future__ import annotations

from dataclasses import dataclass
from typing import Any

import torch
from torch import nn

from saelens_b200.models.sae import (
    SAE,
    SAEConfig,
    TrainCoefficientConfig,
    TrainingSAE,
    TrainingSAEConfig,
    TrainStepInput,
)


def _init_gated(sae: SAE[Any]) -> None:
    for name in ("b_gate", "r_mag", "b_mag"):
        setattr(sae, name, nn.Parameter(torch.zeros(sae.cfg.d_sae, dtype=sae.dtype, device=sae.device)))


def _gated_encode(sae: Any, x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    sae_in = sae.process_sae_in(x)
    # one GEMM feeds both paths: x @ (W * e^r) == (x @ W) * e^r
    base = sae_in @ sae.W_enc
    active = (base + sae.b_gate > 0).to(sae.dtype)
    mag_pre = sae.hook_sae_acts_pre(base * sae.r_mag.exp() + sae.b_mag)
    acts = sae.hook_sae_acts_post(active * sae.activation_fn(mag_pre))
    return acts, mag_pre


@dataclass
class GatedSAEConfig(SAEConfig):
    @classmethod
    def architecture(cls) -> str:
        return "gated"


class GatedSAE(SAE[GatedSAEConfig]):
    b_gate: nn.Parameter
    b_mag: nn.Parameter
    r_mag: nn.Parameter

    def __init__(self, cfg: GatedSAEConfig, use_error_term: bool = False):
        super().__init__(cfg, use_error_term)

    def initialize_weights(self) -> None:
        super().initialize_weights()
        _init_gated(self)

    def encode(self, x: torch.Tensor) -> torch.Tensor:
        return _gated_encode(self, x)[0]

    def decode(self, feature_acts: torch.Tensor) -> torch.Tensor:
        out = self.hook_sae_recons(feature_acts @ self.W_dec + self.b_dec)
        out = self.run_time_activation_norm_fn_out(out)
        return self.reshape_fn_out(out, self.d_head)

    @torch.no_grad()
    def fold_W_dec_norm(self) -> None:
        norms = self.W_dec.norm(dim=-1).clamp(min=1e-8).unsqueeze(1)
        self.W_dec.data = self.W_dec.data / norms
        self.W_enc.data = self.W_enc.data * norms.T
        self.b_gate.data = self.b_gate.data * norms.squeeze()
        self.b_mag.data = self.b_mag.data * norms.squeeze()


@dataclass
class GatedTrainingSAEConfig(TrainingSAEConfig):
    l1_coefficient: float = 1.0
    l1_warm_up_steps: int = 0

    @classmethod
    def architecture(cls) -> str:
        return "gated"


class GatedTrainingSAE(TrainingSAE[GatedTrainingSAEConfig]):
    b_gate: nn.Parameter
    b_mag: nn.Parameter
    r_mag: nn.Parameter

    def __init__(self, cfg: GatedTrainingSAEConfig, use_error_term: bool = False):
        if use_error_term:
            raise ValueError("GatedSAE does not support `use_error_term`. Please set `use_error_term=False`.")
        super().__init__(cfg, use_error_term)

    def initialize_weights(self) -> None:
        super().initialize_weights()
        _init_gated(self)

    def encode_with_hidden_pre(self, x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        return _gated_encode(self, x)

    def calculate_aux_loss(self, step_input: TrainStepInput, feature_acts: torch.Tensor,
                           hidden_pre: torch.Tensor, sae_out: torch.Tensor) -> dict[str, torch.Tensor]:
        centered = step_input.sae_in - self.b_dec * self.cfg.apply_b_dec_to_input
        pi_gate = torch.relu(centered @ self.W_enc + self.b_gate)
        l1 = step_input.coefficients["l1"] * torch.sum(pi_gate * self.W_dec.norm(dim=1), dim=-1).mean()
        via_gate = pi_gate @ self.W_dec + self.b_dec
        aux = (via_gate - step_input.sae_in).pow(2).sum(dim=-1).mean()
        return {"l1_loss": l1, "auxiliary_reconstruction_loss": aux}

    def get_coefficients(self) -> dict[str, float | TrainCoefficientConfig]:
        return {"l1": TrainCoefficientConfig(self.cfg.l1_coefficient, self.cfg.l1_warm_up_steps)}

    def log_histograms(self) -> dict[str, Any]:
        return {
            **super().log_histograms(),
            "weights/b_gate": self.b_gate.detach().float().cpu().numpy(),
            "weights/b_mag": self.b_mag.detach().float().cpu().numpy(),
        }

    @torch.no_grad()
    def fold_W_dec_norm(self) -> None:
        norms = self.W_dec.norm(dim=-1).clamp(min=1e-8).unsqueeze(1)
        self.W_dec.data = self.W_dec.data / norms
        self.W_enc.data = self.W_enc.data * norms.T
        self.b_gate.data = self.b_gate.data * norms.squeeze()
        self.b_mag.data = self.b_mag.data * norms.squeeze()
