"""JumpReLU SAEs (sae_lens/saes/jumprelu_sae.py): `x * 1[x > theta]` with a rectangle-kernel
straight-through estimator for the threshold; training keeps `log_threshold`."""

from __future__ import annotations

from dataclasses import dataclass
from typing import Any, Literal

import math

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


def rectangle(x: torch.Tensor) -> torch.Tensor:
    return ((x > -0.5) & (x < 0.5)).to(x)


class Step(torch.autograd.Function):
    """Heaviside step 1[x > theta]; d/dtheta = -(1/bw) rect((x-theta)/bw)."""

    @staticmethod
    def forward(ctx: Any, x: torch.Tensor, threshold: torch.Tensor, bandwidth: float) -> torch.Tensor:
        ctx.save_for_backward(x, threshold)
        ctx.bandwidth = bandwidth
        return (x > threshold).to(x)

    @staticmethod
    def backward(ctx: Any, g: torch.Tensor) -> tuple[None, torch.Tensor, None]:
        x, th = ctx.saved_tensors
        bw = ctx.bandwidth
        gth = torch.sum(-(1.0 / bw) * rectangle((x - th) / bw) * g, dim=0)
        return None, gth, None


class JumpReLU(torch.autograd.Function):
    """x * 1[x > theta]; d/dx = 1[x > theta], d/dtheta = -(theta/bw) rect((x-theta)/bw)."""

    @staticmethod
    def forward(ctx: Any, x: torch.Tensor, threshold: torch.Tensor, bandwidth: float) -> torch.Tensor:
        ctx.save_for_backward(x, threshold)
        ctx.bandwidth = bandwidth
        return (x * (x > threshold)).to(x)

    @staticmethod
    def backward(ctx: Any, g: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor, None]:
        x, th = ctx.saved_tensors
        bw = ctx.bandwidth
        gx = (x > th) * g
        gth = torch.sum(-(th / bw) * rectangle((x - th) / bw) * g, dim=0)
        return gx, gth, None


@dataclass
class JumpReLUSAEConfig(SAEConfig):
    @classmethod
    def architecture(cls) -> str:
        return "jumprelu"


class JumpReLUSAE(SAE[JumpReLUSAEConfig]):
    b_enc: nn.Parameter
    threshold: nn.Parameter

    def initialize_weights(self) -> None:
        super().initialize_weights()
        self.threshold = nn.Parameter(torch.zeros(self.cfg.d_sae, dtype=self.dtype, device=self.device))
        self.b_enc = nn.Parameter(torch.zeros(self.cfg.d_sae, dtype=self.dtype, device=self.device))

    def encode(self, x: torch.Tensor) -> torch.Tensor:
        sae_in = self.process_sae_in(x)
        pre = self.hook_sae_acts_pre(sae_in @ self.W_enc + self.b_enc)
        acts = self.activation_fn(pre)
        return self.hook_sae_acts_post(acts * (pre > self.threshold).to(acts.dtype))

    def decode(self, feature_acts: torch.Tensor) -> torch.Tensor:
        out = self.hook_sae_recons(feature_acts @ self.W_dec + self.b_dec)
        out = self.run_time_activation_norm_fn_out(out)
        return self.reshape_fn_out(out, self.d_head)

    @torch.no_grad()
    def fold_W_dec_norm(self) -> None:
        th = self.threshold.clone()
        norms = self.W_dec.norm(dim=-1).clamp(min=1e-8)
        super().fold_W_dec_norm()
        self.threshold.data = th * norms


@dataclass
class JumpReLUTrainingSAEConfig(TrainingSAEConfig):
    jumprelu_init_threshold: float = 0.01
    jumprelu_bandwidth: float = 0.05
    jumprelu_sparsity_loss_mode: Literal["step", "tanh"] = "step"
    l0_coefficient: float = 1.0
    l0_warm_up_steps: int = 0
    pre_act_loss_coefficient: float | None = None
    jumprelu_tanh_scale: float = 4.0

    @classmethod
    def architecture(cls) -> str:
        return "jumprelu"


def calculate_pre_act_loss(coef: float, threshold: torch.Tensor, hidden_pre: torch.Tensor,
                           dead_neuron_mask: torch.Tensor | None, W_dec_norm: torch.Tensor) -> torch.Tensor:
    if dead_neuron_mask is None or not dead_neuron_mask.any():
        return hidden_pre.new_tensor(0.0)
    per_item = ((threshold - hidden_pre).relu() * dead_neuron_mask * W_dec_norm).sum(dim=-1)
    return coef * per_item.mean()


class JumpReLUTrainingSAE(TrainingSAE[JumpReLUTrainingSAEConfig]):
    b_enc: nn.Parameter
    log_threshold: nn.Parameter

    def __init__(self, cfg: JumpReLUTrainingSAEConfig, use_error_term: bool = False):
        super().__init__(cfg, use_error_term)
        self.bandwidth = cfg.jumprelu_bandwidth
        self.log_threshold = nn.Parameter(
            torch.ones(cfg.d_sae, dtype=self.dtype, device=self.device) * math.log(cfg.jumprelu_init_threshold)
        )

    def initialize_weights(self) -> None:
        super().initialize_weights()
        self.b_enc = nn.Parameter(torch.zeros(self.cfg.d_sae, dtype=self.dtype, device=self.device))

    @property
    def threshold(self) -> torch.Tensor:
        return torch.exp(self.log_threshold)

    def encode_with_hidden_pre(self, x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        sae_in = self.process_sae_in(x)
        pre = sae_in @ self.W_enc + self.b_enc
        acts = JumpReLU.apply(pre, self.threshold, self.bandwidth)
        return acts, pre  # type: ignore[return-value]

    def calculate_aux_loss(self, step_input: TrainStepInput, feature_acts: torch.Tensor,
                           hidden_pre: torch.Tensor, sae_out: torch.Tensor) -> dict[str, torch.Tensor]:
        th = self.threshold
        wn = self.W_dec.norm(dim=1)
        if self.cfg.jumprelu_sparsity_loss_mode == "step":
            l0 = torch.sum(Step.apply(hidden_pre, th, self.bandwidth), dim=-1)  # type: ignore[arg-type]
            l0_loss = (step_input.coefficients["l0"] * l0).mean()
        elif self.cfg.jumprelu_sparsity_loss_mode == "tanh":
            per = torch.tanh(self.cfg.jumprelu_tanh_scale * feature_acts * wn).sum(dim=-1)
            l0_loss = (step_input.coefficients["l0"] * per).mean()
        else:
            raise ValueError(f"Invalid sparsity loss mode: {self.cfg.jumprelu_sparsity_loss_mode}")
        losses = {"l0_loss": l0_loss}
        if self.cfg.pre_act_loss_coefficient is not None:
            losses["pre_act_loss"] = calculate_pre_act_loss(
                self.cfg.pre_act_loss_coefficient, th, hidden_pre, step_input.dead_neuron_mask, wn,
            )
        return losses

    def get_coefficients(self) -> dict[str, float | TrainCoefficientConfig]:
        return {"l0": TrainCoefficientConfig(self.cfg.l0_coefficient, self.cfg.l0_warm_up_steps)}

    @torch.no_grad()
    def fold_W_dec_norm(self) -> None:
        th = self.threshold.clone()
        norms = self.W_dec.norm(dim=-1).clamp(min=1e-8)
        super().fold_W_dec_norm()
        self.log_threshold.data = torch.log(th * norms)

    def process_state_dict_for_saving(self, state_dict: dict[str, Any]) -> None:
        if "log_threshold" in state_dict:
            state_dict["threshold"] = torch.exp(state_dict.pop("log_threshold")).detach().contiguous()

    def process_state_dict_for_loading(self, state_dict: dict[str, Any]) -> None:
        if "threshold" in state_dict:
            state_dict["log_threshold"] = torch.log(state_dict.pop("threshold")).detach().contiguous()
