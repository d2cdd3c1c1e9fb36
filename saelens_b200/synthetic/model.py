"""SyntheticModel: a serialisable bundle of feature dictionary + activation generator (+ optional
hierarchy and correlation), the toy "language model" of synthetic SAE benchmarks (role of
sae_lens/synthetic/synthetic_model.py, training.py, initialization.py, stats.py).

Saved layout (directory): `synthetic_model_config.json` (the config), `synthetic_model.safetensors`
(feature vectors, bias, firing probabilities, magnitudes, low-rank correlation factors) and, with a
hierarchy, `synthetic_model_hierarchy.json`.
"""

from __future__ import annotations

import json
from collections.abc import Callable, Iterator
from dataclasses import asdict, dataclass, field
from pathlib import Path
from typing import Any

import torch
from torch import nn

from saelens_b200.synthetic.distributions import (
    FiringProbabilityConfig,
    LowRankCorrelationMatrix,
    MagnitudeConfig,
    ZipfianFiringProbabilityConfig,
    generate_magnitudes,
    generate_random_low_rank_correlation_matrix,
)
from saelens_b200.synthetic.generation import (
    ActivationGenerator,
    FeatureDictionary,
    Hierarchy,
    HierarchyConfig,
    generate_hierarchy,
    orthogonal_initializer,
)
from saelens_b200.utils.misc import cosine_similarities

SYNTHETIC_MODEL_CONFIG_FILENAME = "synthetic_model_config.json"
SYNTHETIC_MODEL_WEIGHTS_FILENAME = "synthetic_model.safetensors"
SYNTHETIC_MODEL_HIERARCHY_FILENAME = "synthetic_model_hierarchy.json"


@dataclass
class OrthogonalizationConfig:
    num_steps: int = 200
    lr: float = 0.01
    chunk_size: int = 1024

    def to_dict(self) -> dict[str, Any]:
        return asdict(self)

    @classmethod
    def from_dict(cls, d: dict[str, Any]) -> "OrthogonalizationConfig":
        return cls(**d)


@dataclass
class LowRankCorrelationConfig:
    rank: int = 32
    correlation_scale: float = 0.075

    def to_dict(self) -> dict[str, Any]:
        return asdict(self)

    @classmethod
    def from_dict(cls, d: dict[str, Any]) -> "LowRankCorrelationConfig":
        return cls(**d)


def _mag_to_json(v: float | MagnitudeConfig) -> Any:
    return v.to_dict() if isinstance(v, MagnitudeConfig) else float(v)


def _mag_from_json(v: Any) -> float | MagnitudeConfig:
    return MagnitudeConfig.from_dict(v) if isinstance(v, dict) else float(v)


@dataclass
class SyntheticModelConfig:
    num_features: int = 16384
    hidden_dim: int = 768
    firing_probability: FiringProbabilityConfig = field(default_factory=ZipfianFiringProbabilityConfig)
    mean_firing_magnitude: float | MagnitudeConfig = 1.0
    std_firing_magnitude: float | MagnitudeConfig = 0.0
    bias: bool | float = False
    orthogonalization: OrthogonalizationConfig | None = field(default_factory=OrthogonalizationConfig)
    correlation: LowRankCorrelationConfig | None = None
    hierarchy: HierarchyConfig | None = None
    seed: int = 42
    dtype: str = "float32"

    def __post_init__(self) -> None:
        if self.num_features < 1 or self.hidden_dim < 1:
            raise ValueError("num_features and hidden_dim must be positive")

    def to_dict(self) -> dict[str, Any]:
        return {"num_features": self.num_features, "hidden_dim": self.hidden_dim,
                "firing_probability": self.firing_probability.to_dict(),
                "mean_firing_magnitude": _mag_to_json(self.mean_firing_magnitude),
                "std_firing_magnitude": _mag_to_json(self.std_firing_magnitude), "bias": self.bias,
                "orthogonalization": self.orthogonalization.to_dict() if self.orthogonalization else None,
                "correlation": self.correlation.to_dict() if self.correlation else None,
                "hierarchy": self.hierarchy.to_dict() if self.hierarchy else None, "seed": self.seed,
                "dtype": self.dtype}

    @classmethod
    def from_dict(cls, d: dict[str, Any]) -> "SyntheticModelConfig":
        return cls(num_features=d["num_features"], hidden_dim=d["hidden_dim"],
                   firing_probability=FiringProbabilityConfig.from_dict(d["firing_probability"]),
                   mean_firing_magnitude=_mag_from_json(d.get("mean_firing_magnitude", 1.0)),
                   std_firing_magnitude=_mag_from_json(d.get("std_firing_magnitude", 0.0)),
                   bias=d.get("bias", False),
                   orthogonalization=OrthogonalizationConfig.from_dict(d["orthogonalization"])
                   if d.get("orthogonalization") else None,
                   correlation=LowRankCorrelationConfig.from_dict(d["correlation"]) if d.get("correlation") else None,
                   hierarchy=HierarchyConfig.from_dict(d["hierarchy"]) if d.get("hierarchy") else None,
                   seed=d.get("seed", 42), dtype=d.get("dtype", "float32"))


class SyntheticModel(nn.Module):
    """`sample(batch)` -> hidden activations [batch, hidden_dim]; `sample_with_features(batch)` also
    returns the ground-truth feature activations."""

    def __init__(self, cfg: SyntheticModelConfig, feature_dict: FeatureDictionary | None = None,
                 activation_generator: ActivationGenerator | None = None, hierarchy: Hierarchy | None = None,
                 correlation_matrix: LowRankCorrelationMatrix | None = None, device: str | torch.device = "cpu",
                 _tensors: dict[str, torch.Tensor] | None = None):
        """Built from `cfg` (and its seed); components given explicitly (a feature dictionary, a
        generator, a hierarchy, a low-rank correlation) are used instead of being generated, as in
        sae_lens/synthetic/synthetic_model.py's constructor.  `_tensors` restores saved state."""
        super().__init__()
        self.cfg = cfg
        self.device = torch.device(device)
        _hierarchy = hierarchy
        t = dict(_tensors or {})
        if correlation_matrix is not None:
            t["correlation_factor"] = correlation_matrix.correlation_factor
            t["correlation_diag"] = correlation_matrix.correlation_diag
        init = None
        if feature_dict is None and "feature_vectors" not in t and cfg.orthogonalization is not None:
            o = cfg.orthogonalization
            init = orthogonal_initializer(num_steps=o.num_steps, lr=o.lr, chunk_size=o.chunk_size)
        self.feature_dict = feature_dict if feature_dict is not None else FeatureDictionary(
            cfg.num_features, cfg.hidden_dim, bias=cfg.bias, initializer=init, device=self.device, seed=cfg.seed)
        if feature_dict is None and "feature_vectors" in t:
            with torch.no_grad():
                self.feature_dict.feature_vectors.copy_(t["feature_vectors"])
                self.feature_dict.bias.copy_(t["bias"])
        self.hierarchy = _hierarchy if _hierarchy is not None else (
            generate_hierarchy(cfg.num_features, cfg.hierarchy, seed=cfg.seed) if cfg.hierarchy else None)
        probs = t.get("firing_probabilities")
        if probs is None:
            probs = cfg.firing_probability.generate(cfg.num_features, seed=cfg.seed)
            if self.hierarchy is not None and cfg.hierarchy is not None and cfg.hierarchy.compensate_probabilities:
                probs = (probs * self.hierarchy.compute_probability_correction_factors(probs)).clamp(max=1.0)
        mean = t.get("mean_firing_magnitudes", generate_magnitudes(cfg.num_features, cfg.mean_firing_magnitude,
                                                                   seed=cfg.seed + 1))
        std = t.get("std_firing_magnitudes", generate_magnitudes(cfg.num_features, cfg.std_firing_magnitude,
                                                                 seed=cfg.seed + 2))
        corr = None
        if "correlation_factor" in t:
            corr = LowRankCorrelationMatrix(t["correlation_factor"], t["correlation_diag"])
        elif cfg.correlation is not None:
            corr = generate_random_low_rank_correlation_matrix(cfg.num_features, cfg.correlation.rank,
                                                               cfg.correlation.correlation_scale, seed=cfg.seed + 3)
        self.correlation = corr
        self.activation_generator = activation_generator if activation_generator is not None else ActivationGenerator(
            cfg.num_features, probs, std_firing_magnitudes=std, mean_firing_magnitudes=mean,
            modify_activations=self.hierarchy.modifier if self.hierarchy is not None else None,
            correlation_matrix=corr, device=self.device, dtype=cfg.dtype)

    def to(self, device: str | torch.device | None = None, dtype: torch.dtype | None = None,  # type: ignore[override]
           non_blocking: bool = False) -> "SyntheticModel":
        """Move the model to `device` (dtype is ignored, as in sae_lens/synthetic/synthetic_model.py:
        644-663): the dictionary moves, and the generator is rebuilt there from its current
        probabilities, magnitudes and correlation (plain tensors that Module.to would not move)."""
        if device is None:
            return self
        self.device = torch.device(device)
        self.feature_dict = self.feature_dict.to(self.device)
        g = self.activation_generator
        corr = None
        if self.correlation is not None:
            corr = LowRankCorrelationMatrix(self.correlation.correlation_factor.to(self.device),
                                            self.correlation.correlation_diag.to(self.device))
            self.correlation = corr
        sparse = g.use_sparse_tensors
        self.activation_generator = ActivationGenerator(
            self.cfg.num_features, g.firing_probabilities.to(self.device),
            std_firing_magnitudes=g.std_firing_magnitudes.to(self.device),
            mean_firing_magnitudes=g.mean_firing_magnitudes.to(self.device),
            modify_activations=self.hierarchy.modifier if self.hierarchy is not None else None,
            correlation_matrix=corr, device=self.device, dtype=self.cfg.dtype, use_sparse_tensors=sparse)
        return self

    @property
    def use_sparse_tensors(self) -> bool:
        return self.activation_generator.use_sparse_tensors

    @use_sparse_tensors.setter
    def use_sparse_tensors(self, value: bool) -> None:
        self.activation_generator.use_sparse_tensors = value

    @torch.no_grad()
    def sample_with_features(self, batch_size: int) -> tuple[torch.Tensor, torch.Tensor]:
        f = self.activation_generator.sample(batch_size)
        return self.feature_dict(f), f

    @torch.no_grad()
    def sample(self, batch_size: int) -> torch.Tensor:
        return self.sample_with_features(batch_size)[0]

    def forward(self, batch_size: int) -> torch.Tensor:
        return self.sample(batch_size)

    # ---------------------------------------------------------------------- persistence
    def save(self, path: str | Path) -> None:
        from safetensors.torch import save_file

        p = Path(path)
        p.mkdir(parents=True, exist_ok=True)
        (p / SYNTHETIC_MODEL_CONFIG_FILENAME).write_text(json.dumps(self.cfg.to_dict(), indent=2))
        g = self.activation_generator
        t = {"feature_vectors": self.feature_dict.feature_vectors.detach(), "bias": self.feature_dict.bias.detach(),
             "firing_probabilities": g.firing_probabilities, "mean_firing_magnitudes": g.mean_firing_magnitudes,
             "std_firing_magnitudes": g.std_firing_magnitudes}
        if self.correlation is not None:
            t["correlation_factor"] = self.correlation.correlation_factor
            t["correlation_diag"] = self.correlation.correlation_diag
        save_file({k: v.contiguous().cpu() for k, v in t.items()}, str(p / SYNTHETIC_MODEL_WEIGHTS_FILENAME))
        if self.hierarchy is not None:
            (p / SYNTHETIC_MODEL_HIERARCHY_FILENAME).write_text(json.dumps(self.hierarchy.to_dict()))

    @classmethod
    def load_from_disk(cls, path: str | Path, device: str | torch.device = "cpu") -> "SyntheticModel":
        from safetensors.torch import load_file

        p = Path(path)
        cfg = SyntheticModelConfig.from_dict(json.loads((p / SYNTHETIC_MODEL_CONFIG_FILENAME).read_text()))
        t = {k: v.to(device) for k, v in load_file(str(p / SYNTHETIC_MODEL_WEIGHTS_FILENAME)).items()}
        hp = p / SYNTHETIC_MODEL_HIERARCHY_FILENAME
        h = Hierarchy.from_dict(json.loads(hp.read_text())) if hp.exists() else None
        return cls(cfg, hierarchy=h, device=device, _tensors=t)

    @classmethod
    def from_pretrained(cls, repo_id: str, model_path: str | None = None, device: str | torch.device = "cpu",
                        force_download: bool = False, revision: str | None = None) -> "SyntheticModel":
        """A model saved on the Hugging Face hub, at the repo root or in its `model_path`
        subfolder (sae_lens/synthetic/synthetic_model.py:585-640)."""
        from huggingface_hub import snapshot_download

        root = Path(snapshot_download(repo_id, revision=revision, force_download=force_download,
                                      allow_patterns=[f"{model_path}/*"] if model_path else None))
        return cls.load_from_disk(root / model_path if model_path else root, device=device)

    @classmethod
    def load_from_source(cls, source: str | Path, device: str | torch.device = "cpu") -> "SyntheticModel":
        """A local directory, or `repo_id[/subfolder]` on the Hugging Face hub."""
        if Path(source).exists():
            return cls.load_from_disk(source, device=device)
        parts = str(source).split("/")
        return cls.from_pretrained("/".join(parts[:2]), "/".join(parts[2:]) or None, device=device)


# ---------------------------------------------------------------------------- training helpers
class SyntheticActivationIterator(Iterator[torch.Tensor]):
    """Endless iterator of hidden-activation batches (a data provider): feature activations from an
    ActivationGenerator mapped through a FeatureDictionary (sae_lens/synthetic/training.py:117-165).

    `SyntheticActivationIterator(feature_dict, activations_generator, batch_size, autocast)` as in
    the reference, or `SyntheticActivationIterator(model, batch_size)` with a SyntheticModel.  With
    `autocast` the generator and the dictionary run under bfloat16 autocast; `dtype` / `device`
    cast the served batches."""

    def __init__(self, feature_dict: Any, activations_generator: Any = None, batch_size: int | None = None,
                 autocast: bool = False, dtype: torch.dtype | None = None,
                 device: str | torch.device | None = None):
        if isinstance(activations_generator, int) and batch_size is None:  # (model, batch_size)
            activations_generator, batch_size = None, activations_generator
        if batch_size is None:
            raise TypeError("batch_size is required")
        self.model = feature_dict if activations_generator is None else None
        if self.model is not None:
            feature_dict, activations_generator = self.model.feature_dict, self.model.activation_generator
        self.feature_dict, self.activations_generator = feature_dict, activations_generator
        self.batch_size, self.autocast, self.dtype = int(batch_size), bool(autocast), dtype
        self.device = torch.device(device) if device is not None else feature_dict.feature_vectors.device

    @torch.no_grad()
    def next_batch(self) -> torch.Tensor:
        dev_type = self.feature_dict.feature_vectors.device.type
        with torch.autocast(device_type=dev_type, dtype=torch.bfloat16, enabled=self.autocast):
            if self.model is not None:
                x = self.model.sample(self.batch_size)
            else:
                x = self.feature_dict(self.activations_generator(self.batch_size))
        x = x.to(self.device)
        return x.to(self.dtype) if self.dtype is not None else x

    def __iter__(self) -> "SyntheticActivationIterator":
        return self

    def __next__(self) -> torch.Tensor:
        return self.next_batch()


def init_sae_to_match_feature_dict(sae: Any, feature_dict: FeatureDictionary, noise_level: float = 0.0,
                                   feature_ordering: torch.Tensor | None = None) -> None:
    """Set the SAE decoder rows to the ground-truth features (optionally permuted / noised), the
    encoder to the decoder transpose, and zero the biases."""
    fv = feature_dict.feature_vectors.detach().float()
    if feature_ordering is not None:
        fv = fv[feature_ordering]
    n = min(fv.shape[0], sae.W_dec.shape[0])
    with torch.no_grad():
        W = sae.W_dec.detach().float().clone()
        W[:n] = fv[:n].to(W.device)
        if noise_level > 0:
            W += noise_level * torch.randn_like(W)
        W = W / W.norm(dim=1, keepdim=True).clamp(min=1e-12)
        sae.W_dec.copy_(W.to(sae.W_dec.dtype))
        sae.W_enc.copy_(W.T.to(sae.W_enc.dtype))
        sae.b_enc.zero_()
        sae.b_dec.zero_()


def train_toy_sae(sae: Any, feature_dict: Any, activations_generator: Any = None, training_samples: int = 10_000_000,
                  batch_size: int = 1024, lr: float = 3e-4, lr_warm_up_steps: int = 0, lr_decay_steps: int = 0,
                  device: str | torch.device = "cpu", n_snapshots: int = 0,
                  snapshot_fn: Callable[[Any], None] | None = None, autocast_sae: bool = False,
                  autocast_data: bool = False) -> None:
    """Train `sae` on synthetic activations with the framework's SAETrainer (constant LR with
    optional warm-up / decay, Adam 0.9 / 0.999, no files written): a convenience for small
    experiments (sae_lens/synthetic/training.py:14-114).  `n_snapshots` evenly spaced points call
    `snapshot_fn(trainer)`.  `feature_dict` may also be a SyntheticModel (its dictionary and
    generator are used; `activations_generator` is then omitted)."""
    from saelens_b200.config import LoggingConfig, SAETrainerConfig
    from saelens_b200.training.sae_trainer import SAETrainer

    if n_snapshots > 0 and snapshot_fn is None:
        raise ValueError("snapshot_fn must be provided to take snapshots")
    if activations_generator is None:
        data = SyntheticActivationIterator(feature_dict, batch_size, autocast=autocast_data)
        feature_dict = feature_dict.feature_dict
    else:
        data = SyntheticActivationIterator(feature_dict, activations_generator, batch_size, autocast=autocast_data)
    cfg = SAETrainerConfig(
        n_checkpoints=n_snapshots, checkpoint_path=None, save_final_checkpoint=False, output_path=None,
        save_mse_every_n_steps=0, save_timing_every_n_steps=0, save_memory_every_n_steps=0,
        synchronize_timing=False, multi_sae_backward_order="forward", multi_sae_stats_sync_mode="immediate",
        multi_sae_stats_sync_interval=1, total_training_samples=training_samples, device=str(device),
        autocast=autocast_sae, lr=lr, lr_end=lr, lr_scheduler_name="constant", lr_warm_up_steps=lr_warm_up_steps,
        adam_beta1=0.9, adam_beta2=0.999, lr_decay_steps=lr_decay_steps, n_restart_cycles=1,
        train_batch_size_samples=batch_size, dead_feature_window=1000, feature_sampling_window=2000,
        logger=LoggingConfig(log_to_wandb=False, eval_every_n_wandb_logs=2**31 - 1))
    feature_dict.eval()
    holder: dict[str, Any] = {}

    def on_checkpoint(checkpoint_path: Any = None) -> None:  # noqa: ARG001 - the trainer's callback form
        if snapshot_fn is not None:
            snapshot_fn(holder["trainer"])

    trainer = SAETrainer(cfg, sae, data, save_checkpoint_fn=on_checkpoint)
    holder["trainer"] = trainer
    trainer.fit()


# ---------------------------------------------------------------------------- statistics
@dataclass
class SuperpositionStats:
    """How much the dictionary's directions overlap (sae_lens/synthetic/stats.py:95-110): per
    feature the largest |cos| to any other feature and chosen percentiles of its |cos| to the
    others, their means, and the mean |cos| over all pairs."""

    max_abs_cos_sims: torch.Tensor
    percentile_abs_cos_sims: dict[int, torch.Tensor]
    mean_max_abs_cos_sim: float
    mean_percentile_abs_cos_sim: dict[int, float]
    mean_abs_cos_sim: float
    num_features: int
    hidden_dim: int


@torch.no_grad()
def compute_superposition_stats(feature_dictionary: Any, batch_size: int = 1024,
                                device: str | torch.device | None = None,
                                percentiles: list[int] | None = None) -> SuperpositionStats:
    """`feature_dictionary`: a FeatureDictionary (or its [num_features, hidden_dim] vectors).
    Rows of the cosine matrix are formed `batch_size` at a time; a feature's similarity to itself
    is left out of its maximum, its percentiles and the pair mean."""
    vectors = getattr(feature_dictionary, "feature_vectors", feature_dictionary)
    pct = [95, 99] if percentiles is None else list(percentiles)
    n, d = vectors.shape
    if n < 2:
        raise ValueError("Need at least 2 features to compute superposition stats")
    dev = vectors.device if device is None else torch.device(device)
    unit = vectors.to(dev).float()
    unit = unit / unit.norm(dim=1, keepdim=True).clamp_min(1e-8)
    row_max = torch.empty(n, device=dev)
    row_pct = {p: torch.empty(n, device=dev) for p in pct}
    total = 0.0
    for s0 in range(0, n, batch_size):
        a = (unit[s0 : s0 + batch_size] @ unit.T).abs()
        r = torch.arange(a.shape[0], device=dev)
        self_cols = s0 + r
        total += float(a.sum() - a[r, self_cols].sum())
        a[r, self_cols] = -1.0  # below every |cos|: never the maximum, sorts first
        row_max[s0 : s0 + a.shape[0]] = a.max(dim=1).values
        others = a.sort(dim=1).values[:, 1:]  # drop the self entry; n - 1 values per row
        for p in pct:  # linear interpolation between order statistics (torch.quantile's default)
            pos = (p / 100.0) * (n - 2)
            lo = int(pos)
            hi = min(lo + 1, n - 2)
            w = pos - lo
            row_pct[p][s0 : s0 + a.shape[0]] = others[:, lo] * (1 - w) + others[:, hi] * w
    return SuperpositionStats(
        max_abs_cos_sims=row_max.cpu(), percentile_abs_cos_sims={p: v.cpu() for p, v in row_pct.items()},
        mean_max_abs_cos_sim=float(row_max.mean()),
        mean_percentile_abs_cos_sim={p: float(v.mean()) for p, v in row_pct.items()},
        mean_abs_cos_sim=total / (n * (n - 1)), num_features=n, hidden_dim=d)


@dataclass
class CorrelationMatrixStats:
    """Off-diagonal statistics of a correlation matrix (sae_lens/synthetic/stats.py:9-15)."""

    rms_correlation: float
    mean_correlation: float
    num_features: int


@torch.no_grad()
def compute_correlation_matrix_stats(correlation_matrix: torch.Tensor) -> CorrelationMatrixStats:
    c = correlation_matrix.double()
    n = c.shape[0]
    pairs = n * (n - 1)
    diag = c.diagonal()
    off_sum = float(c.sum() - diag.sum())
    off_sq = float(c.square().sum() - diag.square().sum())
    return CorrelationMatrixStats(rms_correlation=(off_sq / pairs) ** 0.5 if pairs else 0.0,
                                  mean_correlation=off_sum / pairs if pairs else 0.0, num_features=n)


@torch.no_grad()
def compute_low_rank_correlation_matrix_stats(correlation_matrix: LowRankCorrelationMatrix) -> CorrelationMatrixStats:
    """The same statistics for C = F F^T + diag(d) without forming C: its off-diagonal part is
    F F^T minus its diagonal, so sum(C_off) = |F^T 1|^2 - sum_i |F_i|^2 and
    sum(C_off^2) = |F^T F|_F^2 - sum_i |F_i|^4 (O(n r^2) time, O(r^2) memory)."""
    f = correlation_matrix.correlation_factor.double()
    n = f.shape[0]
    pairs = n * (n - 1)
    row_sq = f.square().sum(dim=1)
    off_sum = float(f.sum(dim=0).square().sum() - row_sq.sum())
    off_sq = float((f.T @ f).square().sum() - row_sq.square().sum())
    return CorrelationMatrixStats(rms_correlation=max(off_sq / pairs, 0.0) ** 0.5 if pairs else 0.0,
                                  mean_correlation=off_sum / pairs if pairs else 0.0, num_features=n)
