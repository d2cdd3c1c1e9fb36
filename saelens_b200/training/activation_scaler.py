"""Fixed activation rescaling `x * sqrt(d_in) / E||x||` (sae_lens/training/activation_scaler.py).

The factor is estimated once from the mean row norm of a number of batches and then applied to
every batch the SAE sees (and undone on its outputs).  The estimate accumulates the per-batch mean
norms on the batches' own device and reads the result back once, instead of once per batch.  The
saved form is the reference's `activation_scaler.json` (`{"scaling_factor": value}`).
"""

from __future__ import annotations

import json
from collections.abc import Iterator
from dataclasses import dataclass
from pathlib import Path

import torch


@dataclass
class ActivationScaler:
    scaling_factor: float | None = None

    def scale(self, acts: torch.Tensor) -> torch.Tensor:
        """Multiply by the factor; without an estimate yet, the identity."""
        factor = self.scaling_factor
        if factor is None:
            return acts
        return acts * factor

    def unscale(self, acts: torch.Tensor) -> torch.Tensor:
        """Undo `scale` (the identity without an estimate)."""
        factor = self.scaling_factor
        if factor is None:
            return acts
        return acts / factor

    def __call__(self, acts: torch.Tensor) -> torch.Tensor:
        return self.scale(acts)

    @torch.no_grad()
    def _calculate_mean_norm(self, data_provider: Iterator[torch.Tensor], n_batches_for_norm_estimate: int = 1000) -> float:
        """Mean over `n_batches_for_norm_estimate` batches of each batch's mean row norm."""
        total: torch.Tensor | None = None
        for _ in range(n_batches_for_norm_estimate):
            batch_mean = next(data_provider).float().norm(dim=-1).mean()
            total = batch_mean if total is None else total + batch_mean
        if total is None:
            raise ValueError("the norm estimate needs at least one batch")
        return float(total) / n_batches_for_norm_estimate

    def estimate_scaling_factor(self, d_in: int, data_provider: Iterator[torch.Tensor],
                                n_batches_for_norm_estimate: int = 1000) -> None:
        """Set the factor so that rows have mean norm sqrt(d_in)."""
        mean_norm = self._calculate_mean_norm(data_provider, n_batches_for_norm_estimate)
        self.scaling_factor = float(d_in) ** 0.5 / mean_norm

    def save(self, file_path: str) -> None:
        path = Path(file_path)
        if path.suffix != ".json":
            raise ValueError(f"the activation scaler is saved as JSON; {file_path!r} does not name a .json file")
        path.write_text(json.dumps({"scaling_factor": self.scaling_factor}))

    def load(self, file_path: str | Path) -> None:
        self.scaling_factor = json.loads(Path(file_path).read_text())["scaling_factor"]
