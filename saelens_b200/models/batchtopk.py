"""BatchTopK and Matryoshka BatchTopK SAEs (sae_lens/saes/batchtopk_sae.py,
matryoshka_batchtopk_sae.py).

BatchTopK keeps the top `k * batch` ReLU activations of the whole batch; a global threshold
(fp64 EMA of the smallest kept activation) replaces the batch selection at inference, which is
why both train as TopK-family SAEs and export as JumpReLU SAEs.
"""

from __future__ import annotations

import warnings
from collections.abc import Callable, Iterator
from dataclasses import dataclass, field
from typing import Any

import torch
from torch import nn

from saelens_b200.models.jumprelu import JumpReLUSAEConfig
from saelens_b200.models.sae import SAEConfig, TrainStepInput, TrainStepOutput
from saelens_b200.models.topk import (
    TopKTrainingSAE,
    TopKTrainingSAEConfig,
    _sparse_matmul,
    act_times_W_dec,
    calculate_topk_aux_acts,
)


class BatchTopK(nn.Module):
    def __init__(self, k: float):
        super().__init__()
        self.k = k

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        acts = x.relu()
        flat = acts.flatten()
        n = acts.shape[:-1].numel()
        top = torch.topk(flat, int(self.k * n), dim=-1)
        return torch.zeros_like(flat).scatter(-1, top.indices, top.values).reshape(acts.shape)


@dataclass
class BatchTopKTrainingSAEConfig(TopKTrainingSAEConfig):
    k: float = 100  # type: ignore[assignment]
    topk_threshold_lr: float = 0.01

    @classmethod
    def architecture(cls) -> str:
        return "batchtopk"

    def get_inference_config_class(self) -> type[SAEConfig]:
        return JumpReLUSAEConfig


class BatchTopKTrainingSAE(TopKTrainingSAE):
    topk_threshold: torch.Tensor
    cfg: BatchTopKTrainingSAEConfig  # type: ignore[assignment]

    def __init__(self, cfg: BatchTopKTrainingSAEConfig, use_error_term: bool = False):
        super().__init__(cfg, use_error_term)  # type: ignore[arg-type]
        self.register_buffer("topk_threshold", torch.tensor(0.0, dtype=torch.double, device=self.W_dec.device))

    def get_activation_fn(self) -> Callable[[torch.Tensor], torch.Tensor]:
        return BatchTopK(self.cfg.k)

    def training_forward_pass(self, step_input: TrainStepInput) -> TrainStepOutput:
        out = super().training_forward_pass(step_input)
        self.update_topk_threshold(out.feature_acts)
        out.metrics["topk_threshold"] = self.topk_threshold
        return out

    @torch.no_grad()
    def update_topk_threshold(self, acts_topk: torch.Tensor) -> None:
        pos = acts_topk > 0
        lr = self.cfg.topk_threshold_lr
        with torch.autocast(self.topk_threshold.device.type, enabled=False):
            if pos.any():
                mn = acts_topk[pos].min().to(self.topk_threshold.dtype)
                self.topk_threshold = (1 - lr) * self.topk_threshold + lr * mn

    def process_state_dict_for_saving_inference(self, state_dict: dict[str, Any]) -> None:
        super().process_state_dict_for_saving_inference(state_dict)
        th = state_dict.pop("topk_threshold").item()
        state_dict["threshold"] = torch.ones_like(state_dict["b_enc"]) * th


@dataclass
class MatryoshkaBatchTopKTrainingSAEConfig(BatchTopKTrainingSAEConfig):
    matryoshka_widths: list[int] = field(default_factory=list)
    use_matryoshka_aux_loss: bool = False

    @classmethod
    def architecture(cls) -> str:
        return "matryoshka_batchtopk"


def _validate_matryoshka_config(cfg: MatryoshkaBatchTopKTrainingSAEConfig) -> None:
    if not cfg.matryoshka_widths or cfg.matryoshka_widths[-1] != cfg.d_sae:
        warnings.warn(
            "WARNING: The final matryoshka level width is not set to cfg.d_sae. "
            "A final matryoshka level of width=cfg.d_sae will be added.",
            stacklevel=3,
        )
        cfg.matryoshka_widths.append(cfg.d_sae)
    for a, b in zip(cfg.matryoshka_widths[:-1], cfg.matryoshka_widths[1:]):
        if a >= b:
            raise ValueError("cfg.matryoshka_widths must be strictly increasing.")
    if len(cfg.matryoshka_widths) == 1:
        warnings.warn(
            "WARNING: You have only set one matryoshka level. This is equivalent to using a "
            "standard BatchTopK SAE and is likely not what you want.",
            stacklevel=3,
        )


class MatryoshkaBatchTopKTrainingSAE(BatchTopKTrainingSAE):
    cfg: MatryoshkaBatchTopKTrainingSAEConfig  # type: ignore[assignment]

    def __init__(self, cfg: MatryoshkaBatchTopKTrainingSAEConfig, use_error_term: bool = False):
        super().__init__(cfg, use_error_term)
        _validate_matryoshka_config(cfg)

    def _iterable_decode(self, feature_acts: torch.Tensor,
                         include_outer_loss: bool = False) -> Iterator[tuple[int, torch.Tensor]]:
        if self.cfg.rescale_acts_by_decoder_norm:
            feature_acts = feature_acts * (1 / self.W_dec.norm(dim=-1))
        widths = self.cfg.matryoshka_widths if include_outer_loss else self.cfg.matryoshka_widths[:-1]
        prev = 0
        decoded: torch.Tensor = self.b_dec
        for w in widths:
            part = feature_acts[:, prev:w]
            if part.is_sparse:
                decoded = _sparse_matmul(part, self.W_dec[prev:w]) + decoded
            else:
                decoded = part @ self.W_dec[prev:w] + decoded
            prev = w
            yield w, self.run_time_activation_norm_fn_out(decoded)

    def training_forward_pass(self, step_input: TrainStepInput) -> TrainStepOutput:
        out = super().training_forward_pass(step_input)
        for w, inner in self._iterable_decode(out.feature_acts, include_outer_loss=False):
            l = self.mse_loss_fn(inner, step_input.sae_in).sum(dim=-1).mean()
            out.losses[f"inner_mse_loss_{w}"] = l
            out.loss = out.loss + l
        return out

    def calculate_aux_loss(self, step_input: TrainStepInput, feature_acts: torch.Tensor,
                           hidden_pre: torch.Tensor, sae_out: torch.Tensor) -> dict[str, torch.Tensor]:
        if self.cfg.use_matryoshka_aux_loss:
            aux = self.calculate_matryoshka_aux_loss(step_input.sae_in, sae_out, feature_acts,
                                                     hidden_pre, step_input.dead_neuron_mask)
        else:
            aux = self.calculate_topk_aux_loss(sae_in=step_input.sae_in, sae_out=sae_out,
                                               hidden_pre=hidden_pre,
                                               dead_neuron_mask=step_input.dead_neuron_mask)
        return {"auxiliary_reconstruction_loss": aux}

    def calculate_matryoshka_aux_loss(self, sae_in: torch.Tensor, sae_out: torch.Tensor,
                                      feature_acts: torch.Tensor, hidden_pre: torch.Tensor,
                                      dead_neuron_mask: torch.Tensor | None) -> torch.Tensor:
        if dead_neuron_mask is None or int(dead_neuron_mask.sum()) == 0:
            return sae_out.new_tensor(0.0)
        k_aux = sae_in.shape[-1] // 2
        W = self.W_dec / self.W_dec.norm(dim=-1, keepdim=True) if self.cfg.rescale_acts_by_decoder_norm else self.W_dec
        losses = []
        prev = 0
        for w, partial_out in self._iterable_decode(feature_acts, include_outer_loss=True):
            dmask = dead_neuron_mask[prev:w]
            nd = int(dmask.sum())
            if nd == 0:
                prev = w
                continue
            scale = min(nd / k_aux, 1.0)
            resid = (sae_in - partial_out).detach()
            acts = calculate_topk_aux_acts(min(k_aux, nd), hidden_pre[:, prev:w], dmask)
            rec = act_times_W_dec(acts, W[prev:w], rescale_acts_by_decoder_norm=False)
            losses.append(scale * (rec - resid).pow(2).sum(dim=-1).mean())
            prev = w
        if not losses:
            return sae_out.new_tensor(0.0)
        return self.cfg.aux_loss_coefficient * torch.stack(losses).sum()
