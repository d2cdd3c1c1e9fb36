"""Matching-pursuit SAEs (sae_lens/saes/matching_pursuit_sae.py): greedy encode that repeatedly
picks the decoder row best aligned with the residual; the encoder is tied to W_dec^T.

On CUDA the encode runs natively (`saelens_b200.ops.mp`: the tcgen05 score GEMM with a fused row
argmax, a fused per-row update, and a replaying backward); the loop below is the CPU path and the
test oracle."""

from __future__ import annotations

import warnings
from dataclasses import dataclass
from typing import Any

import torch

from saelens_b200.models.sae import (
    SAE,
    SAEConfig,
    TrainCoefficientConfig,
    TrainingSAE,
    TrainingSAEConfig,
    TrainStepInput,
    TrainStepOutput,
)


def _encode_matching_pursuit(sae_in_centered: torch.Tensor, W_dec: torch.Tensor, residual_threshold: float,
                             max_iterations: int | None, stop_on_duplicate_support: bool) -> torch.Tensor:
    from saelens_b200.ops import mp

    if mp.native_supported(sae_in_centered, W_dec):
        return mp.encode_matching_pursuit(sae_in_centered, W_dec, residual_threshold, max_iterations,
                                          stop_on_duplicate_support)
    return _encode_matching_pursuit_torch(sae_in_centered, W_dec, residual_threshold, max_iterations,
                                          stop_on_duplicate_support)


def _encode_matching_pursuit_torch(sae_in_centered: torch.Tensor, W_dec: torch.Tensor, residual_threshold: float,
                                   max_iterations: int | None, stop_on_duplicate_support: bool,
                                   picks: list[torch.Tensor] | None = None) -> torch.Tensor:
    """PyTorch loop of the reference's iteration.  `picks`, when given, replaces the argmax of
    iteration t by `picks[t]` (a test replays the native kernels' selections this way)."""
    resid = sae_in_centered.clone()
    shape = resid.shape
    if resid.ndim > 2:
        resid = resid.reshape(-1, shape[-1])
    n = resid.shape[0]
    d_sae, d_in = W_dec.shape
    iters = d_in if max_iterations is None else max_iterations
    use_thresh = residual_threshold > 0
    acts = torch.zeros(n, d_sae, device=W_dec.device, dtype=resid.dtype)
    prev = torch.zeros(n, d_sae, dtype=torch.bool, device=W_dec.device)
    done = torch.zeros(n, dtype=torch.bool, device=W_dec.device)
    for it in range(iters):
        if picks is not None and it >= len(picks):
            break
        with torch.no_grad():
            if picks is not None:
                pick = picks[it].to(device=W_dec.device, dtype=torch.int64).clamp_min(0).unsqueeze(1)
            else:
                pick = (resid @ W_dec.T).relu().argmax(dim=1, keepdim=True)
        sel = W_dec[pick.squeeze(1)]
        val = (resid * sel).sum(dim=-1, keepdim=True).relu()
        val = (val * (~done).unsqueeze(1).to(val.dtype)).to(acts.dtype)
        acts = acts.scatter_add(1, pick, val)
        resid = resid - val * sel
        if stop_on_duplicate_support or use_thresh:
            with torch.no_grad():
                support = acts != 0
                if stop_on_duplicate_support:
                    done = done | (support == prev).all(dim=1)
                    prev = support
                if use_thresh:
                    done = done | (resid.norm(dim=-1) < residual_threshold)
                if bool(done.all()):
                    break
    if len(shape) > 2:
        acts = acts.reshape(*shape[:-1], d_sae)
    return acts


class _TiedEncoder:
    """Mixin: W_enc is a read-only view of W_dec^T."""

    @property
    def W_enc(self) -> torch.Tensor:  # type: ignore[override]
        return self.W_dec.T  # type: ignore[attr-defined]

    def __setattr__(self, name: str, value: Any) -> None:
        if name == "W_enc":
            return
        super().__setattr__(name, value)  # type: ignore[misc]


def _mp_decode(sae: Any, feature_acts: torch.Tensor) -> torch.Tensor:
    out = feature_acts @ sae.W_dec
    if sae.cfg.apply_b_dec_to_input:
        out = out + sae.b_dec
    out = sae.hook_sae_recons(out)
    out = sae.run_time_activation_norm_fn_out(out)
    return sae.reshape_fn_out(out, sae.d_head)


@dataclass
class MatchingPursuitSAEConfig(SAEConfig):
    residual_threshold: float = 1e-2
    max_iterations: int | None = None
    stop_on_duplicate_support: bool = True

    @classmethod
    def architecture(cls) -> str:
        return "matching_pursuit"


class MatchingPursuitSAE(_TiedEncoder, SAE[MatchingPursuitSAEConfig]):
    def encode(self, x: torch.Tensor) -> torch.Tensor:
        c = self.cfg
        return _encode_matching_pursuit(self.process_sae_in(x), self.W_dec, c.residual_threshold,
                                        c.max_iterations, c.stop_on_duplicate_support)

    def decode(self, feature_acts: torch.Tensor) -> torch.Tensor:
        return _mp_decode(self, feature_acts)

    @torch.no_grad()
    def fold_W_dec_norm(self) -> None:
        raise NotImplementedError("Folding W_dec_norm is not safe for MatchingPursuit SAEs")


@dataclass
class MatchingPursuitTrainingSAEConfig(TrainingSAEConfig):
    residual_threshold: float = 1e-2
    max_iterations: int | None = None
    stop_on_duplicate_support: bool = True

    @classmethod
    def architecture(cls) -> str:
        return "matching_pursuit"

    def __post_init__(self) -> None:
        super().__post_init__()
        if self.decoder_init_norm != 1.0:
            self.decoder_init_norm = 1.0
            warnings.warn("decoder_init_norm must be set to 1.0 for MatchingPursuitTrainingSAE, setting to 1.0",
                          stacklevel=2)


class MatchingPursuitTrainingSAE(_TiedEncoder, TrainingSAE[MatchingPursuitTrainingSAEConfig]):
    def encode_with_hidden_pre(self, x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        c = self.cfg
        acts = _encode_matching_pursuit(self.process_sae_in(x), self.W_dec, c.residual_threshold,
                                        c.max_iterations, c.stop_on_duplicate_support)
        return acts, torch.zeros_like(acts)

    @torch.no_grad()
    def fold_W_dec_norm(self) -> None:
        raise NotImplementedError("Folding W_dec_norm is not safe for MatchingPursuit SAEs")

    def get_coefficients(self) -> dict[str, float | TrainCoefficientConfig]:
        return {}

    def calculate_aux_loss(self, step_input: TrainStepInput, feature_acts: torch.Tensor,
                           hidden_pre: torch.Tensor, sae_out: torch.Tensor) -> dict[str, torch.Tensor]:
        return {}

    def training_forward_pass(self, step_input: TrainStepInput) -> TrainStepOutput:
        out = super().training_forward_pass(step_input)
        if step_input.is_logging_step:
            l0 = out.feature_acts.bool().float().sum(-1)
            rn = (step_input.sae_in - out.sae_out).norm(dim=-1)
            out.metrics["max_l0"] = l0.max()
            out.metrics["min_l0"] = l0.min()
            out.metrics["residual_norm"] = rn.mean()
            out.metrics["residual_threshold_converged_portion"] = (rn < self.cfg.residual_threshold).float().mean()
        return out

    def decode(self, feature_acts: torch.Tensor) -> torch.Tensor:
        return _mp_decode(self, feature_acts)
