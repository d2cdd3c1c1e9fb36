"""Fixed activation rescaling `x * sqrt(d_in) / E||x||` (sae_lens/training/activation_scaler.py)."""

from __future__ import annotations

import json
from dataclasses import dataclass
from pathlib import Path
from statistics import mean
from collections.abc import Iterator

import torch


@dataclass
class ActivationScaler:
    scaling_factor: float | None = None

    def scale(self, acts: torch.Tensor) -> torch.Tensor:
        return acts if self.scaling_factor is None else acts * self.scaling_factor

    def unscale(self, acts: torch.Tensor) -> torch.Tensor:
        return acts if self.scaling_factor is None else acts / self.scaling_factor

    def __call__(self, acts: torch.Tensor) -> torch.Tensor:
        return self.scale(acts)

    @torch.no_grad()
    def _calculate_mean_norm(self, data_provider: Iterator[torch.Tensor], n_batches_for_norm_estimate: int = 1000) -> float:
        return mean(next(data_provider).float().norm(dim=-1).mean().item() for _ in range(n_batches_for_norm_estimate))

    def estimate_scaling_factor(self, d_in: int, data_provider: Iterator[torch.Tensor],
                                n_batches_for_norm_estimate: int = 1000) -> None:
        self.scaling_factor = (d_in ** 0.5) / self._calculate_mean_norm(data_provider, n_batches_for_norm_estimate)

    def save(self, file_path: str) -> None:
        if not str(file_path).endswith(".json"):
            raise ValueError("file_path must end with .json")
        with open(file_path, "w") as f:
            json.dump({"scaling_factor": self.scaling_factor}, f)

    def load(self, file_path: str | Path) -> None:
        with open(file_path) as f:
            self.scaling_factor = json.load(f)["scaling_factor"]
