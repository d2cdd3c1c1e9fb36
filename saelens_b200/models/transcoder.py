"""Transcoders (sae_lens/saes/transcoder.py): map one hook point to another, d_out may differ
from d_in.  Skip variants add `x @ W_skip^T`; JumpReLU variants threshold the activations."""

from __future__ import annotations

from dataclasses import dataclass
from typing import Any

import torch
from torch import nn

from saelens_b200.models.sae import SAE, SAEConfig, SAEMetadata
from saelens_b200.utils.misc import filter_valid_dataclass_fields


@dataclass
class TranscoderConfig(SAEConfig):
    d_out: int = 768

    @classmethod
    def architecture(cls) -> str:
        return "transcoder"

    @classmethod
    def from_dict(cls, config_dict: dict[str, Any]) -> TranscoderConfig:  # type: ignore[override]
        res = cls(**filter_valid_dataclass_fields(config_dict, cls))
        if "metadata" in config_dict:
            res.metadata = SAEMetadata(**config_dict["metadata"])
        return res

    def __post_init__(self) -> None:
        if self.apply_b_dec_to_input:
            raise ValueError("apply_b_dec_to_input is not supported for transcoders")
        super().__post_init__()


class Transcoder(SAE[TranscoderConfig]):
    b_enc: nn.Parameter

    def __init__(self, cfg: TranscoderConfig):
        super().__init__(cfg)

    def initialize_weights(self) -> None:
        c = self.cfg
        self.b_dec = nn.Parameter(torch.zeros(c.d_out, dtype=self.dtype, device=self.device))
        wd = torch.empty(c.d_sae, c.d_out, dtype=self.dtype, device=self.device)
        nn.init.kaiming_uniform_(wd)
        self.W_dec = nn.Parameter(wd)
        we = torch.empty(c.d_in, c.d_sae, dtype=self.dtype, device=self.device)
        nn.init.kaiming_uniform_(we)
        self.W_enc = nn.Parameter(we)
        self.b_enc = nn.Parameter(torch.zeros(c.d_sae, dtype=self.dtype, device=self.device))

    def process_sae_in(self, sae_in: torch.Tensor) -> torch.Tensor:
        # b_dec lives in the output space, so it is never subtracted from the input
        sae_in = self.hook_sae_input(sae_in.to(self.dtype))
        return self.run_time_activation_norm_fn_in(sae_in)

    def encode(self, x: torch.Tensor) -> torch.Tensor:
        pre = self.hook_sae_acts_pre(self.process_sae_in(x) @ self.W_enc + self.b_enc)
        return self.hook_sae_acts_post(self.activation_fn(pre))

    def decode(self, feature_acts: torch.Tensor) -> torch.Tensor:
        return self.hook_sae_recons(feature_acts @ self.W_dec + self.b_dec)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return self.decode(self.encode(x))

    def forward_with_activations(self, x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        acts = self.encode(x)
        return self.decode(acts), acts

    @property
    def d_out(self) -> int:
        return self.cfg.d_out

    @classmethod
    def from_dict(cls, config_dict: dict[str, Any]) -> Transcoder:  # type: ignore[override]
        return cls(cls._config_cls().from_dict(config_dict))

    @classmethod
    def _config_cls(cls) -> type[TranscoderConfig]:
        return TranscoderConfig


@dataclass
class SkipTranscoderConfig(TranscoderConfig):
    @classmethod
    def architecture(cls) -> str:
        return "skip_transcoder"


class SkipTranscoder(Transcoder):
    W_skip: nn.Parameter

    def __init__(self, cfg: SkipTranscoderConfig):
        super().__init__(cfg)
        self.W_skip = nn.Parameter(torch.zeros(cfg.d_out, cfg.d_in, dtype=self.dtype, device=self.device))

    def _skip(self, x: torch.Tensor) -> torch.Tensor:
        return x @ self.W_skip.T.to(x.device)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return self.decode(self.encode(x)) + self._skip(x)

    def forward_with_activations(self, x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        acts = self.encode(x)
        return self.decode(acts) + self._skip(x), acts

    @classmethod
    def _config_cls(cls) -> type[TranscoderConfig]:
        return SkipTranscoderConfig


@dataclass
class JumpReLUTranscoderConfig(TranscoderConfig):
    @classmethod
    def architecture(cls) -> str:
        return "jumprelu_transcoder"


class JumpReLUTranscoder(Transcoder):
    threshold: nn.Parameter

    def __init__(self, cfg: JumpReLUTranscoderConfig):
        super().__init__(cfg)

    def initialize_weights(self) -> None:
        super().initialize_weights()
        self.threshold = nn.Parameter(torch.zeros(self.cfg.d_sae, dtype=self.dtype, device=self.device))

    def encode(self, x: torch.Tensor) -> torch.Tensor:
        pre = self.hook_sae_acts_pre(self.process_sae_in(x) @ self.W_enc + self.b_enc)
        th = self.threshold.detach() if self.training else self.threshold
        return self.hook_sae_acts_post(self.activation_fn(pre) * (pre > th).to(self.dtype))

    def fold_W_dec_norm(self) -> None:
        with torch.no_grad():
            norms = self.W_dec.norm(dim=1)
        super().fold_W_dec_norm()
        with torch.no_grad():
            self.threshold.data = self.threshold.data * norms

    @classmethod
    def _config_cls(cls) -> type[TranscoderConfig]:
        return JumpReLUTranscoderConfig


@dataclass
class JumpReLUSkipTranscoderConfig(JumpReLUTranscoderConfig):
    @classmethod
    def architecture(cls) -> str:
        return "jumprelu_skip_transcoder"


class JumpReLUSkipTranscoder(JumpReLUTranscoder, SkipTranscoder):
    def __init__(self, cfg: JumpReLUSkipTranscoderConfig):
        super().__init__(cfg)

    @classmethod
    def _config_cls(cls) -> type[TranscoderConfig]:
        return JumpReLUSkipTranscoderConfig
