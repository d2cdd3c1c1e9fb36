"""Per-feature firing probabilities, firing magnitudes and correlation structures for synthetic
SAE benchmarks (roles of sae_lens/synthetic/firing_probabilities.py, firing_magnitudes.py,
correlation.py).

Probability and magnitude generators are small config dataclasses registered by name, so a
synthetic model config can be saved as JSON and rebuilt.  Correlations between feature firings
use a Gaussian copula: a feature fires when its latent Gaussian exceeds the threshold that gives
its marginal firing probability; the latent Gaussians carry either a full correlation matrix or
a low-rank-plus-diagonal one (O(n * rank) memory for millions of features).
"""

from __future__ import annotations

import math
from abc import ABC, abstractmethod
from dataclasses import asdict, dataclass
from typing import Any, NamedTuple

import torch

from saelens_b200.utils.misc import str_to_dtype


class _Registry:
    def __init__(self, kind: str):
        self.kind = kind
        self.items: dict[str, type] = {}

    def register(self, name: str, cls: type) -> None:
        if name in self.items and self.items[name] is not cls:
            raise ValueError(f"'{name}' is already registered.")
        self.items[name] = cls

    def get(self, name: str) -> type:
        if name not in self.items:
            raise ValueError(f"unknown {self.kind} generator {name!r}; known: {sorted(self.items)}")
        return self.items[name]


_PROB = _Registry("firing probability")
_MAG = _Registry("magnitude")


def _generator_name(d: dict[str, Any]) -> str:
    """The registered name in a serialised generator config: "generator_name" (the format the
    reference writes), or "generator" (earlier files of this package)."""
    name = d.get("generator_name", d.get("generator"))
    if name is None:
        raise ValueError("generator_name required in config dict")
    return str(name)


def _fields(d: dict[str, Any]) -> dict[str, Any]:
    return {k: v for k, v in d.items() if k not in ("generator_name", "generator")}


def _register(registry: _Registry, name_or_class: str | type, config_class: type | None) -> Any:
    """register(name, cls) as the reference's API, or @register / register(cls) using the class's
    generator_name(); returns the class (so the one-argument form works as a decorator)."""
    if isinstance(name_or_class, str):
        if config_class is None:
            raise TypeError("register(name, config_class) needs the config class")
        registry.register(name_or_class, config_class)
        return config_class
    registry.register(name_or_class.generator_name(), name_or_class)
    return name_or_class


# ------------------------------------------------------------------------------ probabilities
def zipfian_firing_probabilities(num_features: int, exponent: float = 1.0, max_prob: float = 0.3,
                                 min_prob: float = 0.01) -> torch.Tensor:
    """p_i proportional to 1 / rank^exponent, affinely mapped onto [min_prob, max_prob] (descending)."""
    if num_features < 1:
        raise ValueError("num_features must be at least 1")
    if exponent <= 0:
        raise ValueError("exponent must be positive")
    if not 0 < min_prob < max_prob <= 1:
        raise ValueError("Must have 0 < min_prob < max_prob <= 1")
    if num_features == 1:
        return torch.tensor([max_prob])
    w = torch.arange(1, num_features + 1, dtype=torch.float64).pow(-exponent)
    w = (w - w[-1]) / (w[0] - w[-1])
    return (min_prob + (max_prob - min_prob) * w).float()


def linear_firing_probabilities(num_features: int, max_prob: float = 0.3, min_prob: float = 0.01) -> torch.Tensor:
    if num_features < 1:
        raise ValueError("num_features must be at least 1")
    if not 0 < min_prob <= max_prob <= 1:
        raise ValueError("Must have 0 < min_prob <= max_prob <= 1")
    if num_features == 1:
        return torch.tensor([max_prob])
    return torch.linspace(max_prob, min_prob, num_features)


def random_firing_probabilities(num_features: int, max_prob: float = 0.5, min_prob: float = 0.01,
                                seed: int | None = None) -> torch.Tensor:
    if num_features < 1:
        raise ValueError("num_features must be at least 1")
    if not 0 < min_prob < max_prob <= 1:
        raise ValueError("Must have 0 < min_prob < max_prob <= 1")
    g = torch.Generator()
    if seed is not None:
        g.manual_seed(seed)
    return min_prob + (max_prob - min_prob) * torch.rand(num_features, generator=g)


class FiringProbabilityConfig(ABC):
    """A named generator of per-feature firing probabilities (serialisable)."""

    @classmethod
    @abstractmethod
    def generator_name(cls) -> str: ...

    @abstractmethod
    def generate(self, num_features: int, seed: int | None = None) -> torch.Tensor: ...

    def to_dict(self) -> dict[str, Any]:
        return {**asdict(self), "generator_name": self.generator_name()}  # type: ignore[call-overload]

    @classmethod
    def from_dict(cls, d: dict[str, Any]) -> "FiringProbabilityConfig":
        return _PROB.get(_generator_name(d))(**_fields(d))


def register_firing_probability(name_or_class: str | type, config_class: type | None = None) -> Any:
    return _register(_PROB, name_or_class, config_class)


def get_firing_probability_class(name: str) -> type:
    return _PROB.get(name)


@register_firing_probability
@dataclass
class ZipfianFiringProbabilityConfig(FiringProbabilityConfig):
    exponent: float = 1.0
    max_prob: float = 0.3
    min_prob: float = 0.01

    @classmethod
    def generator_name(cls) -> str:
        return "zipfian"

    def generate(self, num_features: int, seed: int | None = None) -> torch.Tensor:
        return zipfian_firing_probabilities(num_features, self.exponent, self.max_prob, self.min_prob)


@register_firing_probability
@dataclass
class LinearFiringProbabilityConfig(FiringProbabilityConfig):
    max_prob: float = 0.3
    min_prob: float = 0.01

    @classmethod
    def generator_name(cls) -> str:
        return "linear"

    def generate(self, num_features: int, seed: int | None = None) -> torch.Tensor:
        return linear_firing_probabilities(num_features, self.max_prob, self.min_prob)


@register_firing_probability
@dataclass
class RandomFiringProbabilityConfig(FiringProbabilityConfig):
    max_prob: float = 0.5
    min_prob: float = 0.01

    @classmethod
    def generator_name(cls) -> str:
        return "random"

    def generate(self, num_features: int, seed: int | None = None) -> torch.Tensor:
        return random_firing_probabilities(num_features, self.max_prob, self.min_prob, seed)


@register_firing_probability
@dataclass
class ConstantFiringProbabilityConfig(FiringProbabilityConfig):
    probability: float = 0.05

    @classmethod
    def generator_name(cls) -> str:
        return "constant"

    def generate(self, num_features: int, seed: int | None = None) -> torch.Tensor:
        if not 0 < self.probability <= 1:
            raise ValueError("probability must be in (0, 1]")
        return torch.full((num_features,), float(self.probability))


# ------------------------------------------------------------------------------ magnitudes
class MagnitudeConfig(ABC):
    """A named generator of per-feature magnitude values (means or standard deviations)."""

    @classmethod
    @abstractmethod
    def generator_name(cls) -> str: ...

    @abstractmethod
    def generate(self, num_features: int, seed: int | None = None) -> torch.Tensor: ...

    def to_dict(self) -> dict[str, Any]:
        return {**asdict(self), "generator_name": self.generator_name()}  # type: ignore[call-overload]

    @classmethod
    def from_dict(cls, d: dict[str, Any]) -> "MagnitudeConfig":
        return _MAG.get(_generator_name(d))(**_fields(d))


def register_magnitude(name_or_class: str | type, config_class: type | None = None) -> Any:
    return _register(_MAG, name_or_class, config_class)


def get_magnitude_class(name: str) -> type:
    return _MAG.get(name)


def generate_magnitudes(num_features: int, config: float | MagnitudeConfig, seed: int | None = None) -> torch.Tensor:
    if isinstance(config, (int, float)):
        return torch.full((num_features,), float(config))
    return config.generate(num_features, seed=seed)


@register_magnitude
@dataclass
class ConstantMagnitudeConfig(MagnitudeConfig):
    value: float = 1.0

    @classmethod
    def generator_name(cls) -> str:
        return "constant"

    def generate(self, num_features: int, seed: int | None = None) -> torch.Tensor:
        return torch.full((num_features,), float(self.value))


@register_magnitude
@dataclass
class LinearMagnitudeConfig(MagnitudeConfig):
    start: float = 1.0
    end: float = 1.0

    def __post_init__(self) -> None:
        if self.start <= 0 or self.end <= 0:
            raise ValueError("start and end must be positive")

    @classmethod
    def generator_name(cls) -> str:
        return "linear"

    def generate(self, num_features: int, seed: int | None = None) -> torch.Tensor:
        if num_features == 1:
            return torch.tensor([self.start])
        return torch.linspace(self.start, self.end, num_features)


@register_magnitude
@dataclass
class ExponentialMagnitudeConfig(MagnitudeConfig):
    start: float = 1.0
    end: float = 1.0

    def __post_init__(self) -> None:
        if self.start <= 0 or self.end <= 0:
            raise ValueError("start and end must be positive for exponential scale")

    @classmethod
    def generator_name(cls) -> str:
        return "exponential"

    def generate(self, num_features: int, seed: int | None = None) -> torch.Tensor:
        if num_features == 1:
            return torch.tensor([self.start])
        t = torch.linspace(0.0, 1.0, num_features, dtype=torch.float64)
        return (math.log(self.start) + t * (math.log(self.end) - math.log(self.start))).exp().float()


@register_magnitude
@dataclass
class FoldedNormalMagnitudeConfig(MagnitudeConfig):
    """|N(mean, std^2)| per feature, optionally clamped to [min_value, max_value]."""

    mean: float = 0.0
    std: float = 0.1
    min_value: float | None = None
    max_value: float | None = None

    def __post_init__(self) -> None:
        if self.std <= 0:
            raise ValueError("std must be positive")
        if self.min_value is not None and self.min_value < 0:
            raise ValueError("min_value must be non-negative")
        if self.max_value is not None and self.max_value <= 0:
            raise ValueError("max_value must be positive")
        if self.min_value is not None and self.max_value is not None and self.min_value > self.max_value:
            raise ValueError("min_value must be <= max_value")

    @classmethod
    def generator_name(cls) -> str:
        return "folded_normal"

    def generate(self, num_features: int, seed: int | None = None) -> torch.Tensor:
        g = torch.Generator()
        if seed is not None:
            g.manual_seed(seed)
        x = (self.mean + self.std * torch.randn(num_features, generator=g)).abs()
        if self.min_value is not None or self.max_value is not None:
            x = x.clamp(min=self.min_value, max=self.max_value)
        return x


# ------------------------------------------------------------------------------ correlations
class LowRankCorrelationMatrix(NamedTuple):
    """correlation = correlation_factor @ correlation_factor.T + diag(correlation_diag)."""

    correlation_factor: torch.Tensor
    correlation_diag: torch.Tensor


def _nearest_valid_correlation(m: torch.Tensor, min_eig: float = 1e-6) -> torch.Tensor:
    """Clip eigenvalues to be positive and renormalise to a unit diagonal."""
    vals, vecs = torch.linalg.eigh(m)
    fixed = vecs @ torch.diag(vals.clamp(min=min_eig)) @ vecs.T
    d = fixed.diagonal().clamp(min=1e-8).sqrt()
    fixed = fixed / (d[:, None] * d[None, :])
    fixed.fill_diagonal_(1.0)
    return fixed


def _valid_or_fixed(m: torch.Tensor) -> torch.Tensor:
    m = (m + m.T) / 2
    if torch.linalg.eigvalsh(m.double()).min() < -1e-6:
        m = _nearest_valid_correlation(m)
    return m


def create_correlation_matrix_from_correlations(num_features: int,
                                                correlations: dict[tuple[int, int], float] | None = None,
                                                default_correlation: float = 0.0) -> torch.Tensor:
    m = torch.full((num_features, num_features), float(default_correlation))
    m.fill_diagonal_(1.0)
    for (i, j), c in (correlations or {}).items():
        m[i, j] = m[j, i] = c
    return _valid_or_fixed(m)


def _check_corr_params(positive_ratio: float, uncorrelated_ratio: float, lo: float, hi: float) -> None:
    if not 0.0 <= positive_ratio <= 1.0:
        raise ValueError("positive_ratio must be between 0.0 and 1.0")
    if not 0.0 <= uncorrelated_ratio <= 1.0:
        raise ValueError("uncorrelated_ratio must be between 0.0 and 1.0")
    if lo < 0 or hi > 1 or lo > hi:
        raise ValueError("need 0 <= min_correlation_strength <= max_correlation_strength <= 1")


def generate_random_correlations(num_features: int, positive_ratio: float = 0.5, uncorrelated_ratio: float = 0.3,
                                 min_correlation_strength: float = 0.1, max_correlation_strength: float = 0.8,
                                 seed: int | None = None) -> dict[tuple[int, int], float]:
    """Random pairwise correlations {(i, j): c} with i < j (pairs left out are uncorrelated)."""
    _check_corr_params(positive_ratio, uncorrelated_ratio, min_correlation_strength, max_correlation_strength)
    g = torch.Generator()
    if seed is not None:
        g.manual_seed(seed)
    out: dict[tuple[int, int], float] = {}
    if num_features < 2:
        return out
    i, j = torch.triu_indices(num_features, num_features, offset=1)
    keep = torch.rand(i.numel(), generator=g) >= uncorrelated_ratio
    sign = torch.where(torch.rand(i.numel(), generator=g) < positive_ratio, 1.0, -1.0)
    mag = min_correlation_strength + (max_correlation_strength - min_correlation_strength) * torch.rand(
        i.numel(), generator=g)
    for a, b, c in zip(i[keep].tolist(), j[keep].tolist(), (sign * mag)[keep].tolist()):
        out[(a, b)] = c
    return out


def generate_random_correlation_matrix(num_features: int, positive_ratio: float = 0.5, uncorrelated_ratio: float = 0.3,
                                       min_correlation_strength: float = 0.1, max_correlation_strength: float = 0.8,
                                       seed: int | None = None, device: torch.device | str = "cpu",
                                       dtype: torch.dtype | str = torch.float32) -> torch.Tensor:
    _check_corr_params(positive_ratio, uncorrelated_ratio, min_correlation_strength, max_correlation_strength)
    dt = str_to_dtype(dtype) if isinstance(dtype, str) else dtype
    if num_features <= 1:
        return torch.eye(num_features, device=device, dtype=dt)
    g = torch.Generator()
    if seed is not None:
        g.manual_seed(seed)
    i, j = torch.triu_indices(num_features, num_features, offset=1)
    n = i.numel()
    keep = (torch.rand(n, generator=g) >= uncorrelated_ratio).float()
    sign = torch.where(torch.rand(n, generator=g) < positive_ratio, 1.0, -1.0)
    mag = min_correlation_strength + (max_correlation_strength - min_correlation_strength) * torch.rand(n, generator=g)
    m = torch.eye(num_features)
    m[i, j] = keep * sign * mag
    m[j, i] = m[i, j]
    return _valid_or_fixed(m).to(device=device, dtype=dt)


def generate_random_low_rank_correlation_matrix(num_features: int, rank: int, correlation_scale: float = 0.075,
                                                seed: int | None = None, device: torch.device | str = "cpu",
                                                dtype: torch.dtype | str = torch.float32) -> LowRankCorrelationMatrix:
    """Random factor F (n x rank) with entries N(0, correlation_scale^2); diag = 1 - rowsum(F^2)
    so the implied correlation has a unit diagonal (rows whose factor norm would exceed 1 are
    shrunk)."""
    if rank < 1:
        raise ValueError("rank must be at least 1")
    if correlation_scale < 0:
        raise ValueError("correlation_scale must be non-negative")
    dt = str_to_dtype(dtype) if isinstance(dtype, str) else dtype
    g = torch.Generator()
    if seed is not None:
        g.manual_seed(seed)
    f = torch.randn(num_features, rank, generator=g) * correlation_scale
    norm2 = f.square().sum(1)
    too_big = norm2 > 0.99
    if too_big.any():
        f[too_big] *= (0.99 / norm2[too_big]).sqrt()[:, None]
        norm2 = f.square().sum(1)
    return LowRankCorrelationMatrix(f.to(device=device, dtype=dt), (1.0 - norm2).to(device=device, dtype=dt))


def correlation_thresholds(firing_probabilities: torch.Tensor) -> torch.Tensor:
    """Gaussian thresholds t_i with P(N(0,1) > t_i) = p_i (the copula's marginal cut)."""
    return math.sqrt(2.0) * torch.erfinv(1.0 - 2.0 * firing_probabilities.clamp(1e-12, 1 - 1e-7))
