"""Standard ReLU SAE with the decoder-norm-weighted Lp sparsity penalty
(sae_lens/saes/standard_sae.py)."""

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


@dataclass
class StandardSAEConfig(SAEConfig):
    @classmethod
    def architecture(cls) -> str:
        return "standard"


def _zeros_b_enc(sae: SAE[Any]) -> None:
    sae.b_enc = nn.Parameter(torch.zeros(sae.cfg.d_sae, dtype=sae.dtype, device=sae.device))


class StandardSAE(SAE[StandardSAEConfig]):
    b_enc: nn.Parameter

    def initialize_weights(self) -> None:
        super().initialize_weights()
        _zeros_b_enc(self)

    def encode(self, x: torch.Tensor) -> torch.Tensor:
        sae_in = self.process_sae_in(x)
        pre = self.hook_sae_acts_pre(sae_in @ self.W_enc + self.b_enc)
        return self.hook_sae_acts_post(self.activation_fn(pre))

    def decode(self, feature_acts: torch.Tensor) -> torch.Tensor:
        out = self.hook_sae_recons(feature_acts @ self.W_dec + self.b_dec)
        out = self.run_time_activation_norm_fn_out(out)
        return self.reshape_fn_out(out, self.d_head)


@dataclass
class StandardTrainingSAEConfig(TrainingSAEConfig):
    l1_coefficient: float = 1.0
    lp_norm: float = 1.0
    l1_warm_up_steps: int = 0

    @classmethod
    def architecture(cls) -> str:
        return "standard"


class StandardTrainingSAE(TrainingSAE[StandardTrainingSAEConfig]):
    b_enc: nn.Parameter

    def initialize_weights(self) -> None:
        super().initialize_weights()
        _zeros_b_enc(self)

    def get_coefficients(self) -> dict[str, float | TrainCoefficientConfig]:
        return {"l1": TrainCoefficientConfig(self.cfg.l1_coefficient, self.cfg.l1_warm_up_steps)}

    def encode_with_hidden_pre(self, x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        sae_in = self.process_sae_in(x)
        pre = self.hook_sae_acts_pre(sae_in @ self.W_enc + self.b_enc)
        return self.hook_sae_acts_post(self.activation_fn(pre)), pre

    def calculate_aux_loss(self, step_input: TrainStepInput, feature_acts: torch.Tensor,
                           hidden_pre: torch.Tensor, sae_out: torch.Tensor) -> dict[str, torch.Tensor]:
        weighted = feature_acts * self.W_dec.norm(dim=1)
        sparsity = weighted.norm(p=self.cfg.lp_norm, dim=-1)
        return {"l1_loss": (step_input.coefficients["l1"] * sparsity).mean()}

    def log_histograms(self) -> dict[str, Any]:
        return {**super().log_histograms(), "weights/b_e": self.b_enc.detach().float().cpu().numpy()}
