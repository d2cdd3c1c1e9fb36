"""Train an SAE on a SyntheticModel's activations and evaluate it against the ground truth (role
of sae_lens/synthetic/synthetic_sae_runner.py, plotting.py, upload_synthetic_model.py).

The runner reuses SAETrainer, so a TopK SAE on CUDA trains on the fused native engine and every
architecture in the registry is supported; evaluation uses `eval_sae_on_synthetic_data`.
"""

from __future__ import annotations

from collections.abc import Iterable

import json
from dataclasses import asdict, dataclass, field
from pathlib import Path
from typing import Any

import torch

from saelens_b200.config import LoggingConfig, SAETrainerConfig
from saelens_b200.synthetic.evals import SyntheticDataEvalResult, eval_sae_on_synthetic_data
from saelens_b200.synthetic.model import SyntheticActivationIterator, SyntheticModel, SyntheticModelConfig
from saelens_b200.utils.misc import cosine_similarities

RUNNER_CONFIG_FILENAME = "synthetic_runner_config.json"


@dataclass
class SyntheticSAERunnerConfig:
    sae: Any  # a TrainingSAEConfig of any registered architecture
    synthetic_model: SyntheticModelConfig | str | None = None  # config, path or hub id
    training_samples: int = 10_000_000
    train_batch_size_samples: int = 4096
    lr: float = 3e-4
    lr_end: float | None = None
    lr_scheduler_name: str = "constant"
    lr_warm_up_steps: int = 0
    lr_decay_steps: int = 0
    adam_beta1: float = 0.9
    adam_beta2: float = 0.999
    dead_feature_window: int = 1000
    feature_sampling_window: int = 2000
    eval_samples: int = 500_000
    device: str = "cuda" if torch.cuda.is_available() else "cpu"
    output_path: str | None = None
    n_checkpoints: int = 0
    checkpoint_path: str | None = None
    autocast: bool = False
    logger: LoggingConfig = field(default_factory=lambda: LoggingConfig(log_to_wandb=False))
    seed: int = 42

    def __post_init__(self) -> None:
        if self.lr_end is None:
            self.lr_end = self.lr / 10
        if self.training_samples < self.train_batch_size_samples:
            raise ValueError("training_samples must be at least one batch")

    @property
    def total_training_steps(self) -> int:
        return self.training_samples // self.train_batch_size_samples

    def to_dict(self) -> dict[str, Any]:
        d = {k: v for k, v in asdict(self).items() if k not in ("sae", "synthetic_model", "logger")}
        d["sae"] = {"architecture": self.sae.architecture(), **self.sae.to_dict()}
        d["synthetic_model"] = (self.synthetic_model.to_dict() if isinstance(self.synthetic_model, SyntheticModelConfig)
                                else self.synthetic_model)
        return d

    @classmethod
    def from_dict(cls, d: dict[str, Any]) -> "SyntheticSAERunnerConfig":
        from saelens_b200.registry import get_sae_training_class

        d = dict(d)
        sae_d = dict(d.pop("sae"))
        arch = sae_d.pop("architecture")
        _, cfg_cls = get_sae_training_class(arch)
        sm = d.pop("synthetic_model", None)
        return cls(sae=cfg_cls.from_dict(sae_d), synthetic_model=SyntheticModelConfig.from_dict(sm)
                   if isinstance(sm, dict) else sm, **d)

    def to_sae_trainer_config(self) -> SAETrainerConfig:
        return SAETrainerConfig(
            n_checkpoints=self.n_checkpoints, checkpoint_path=self.checkpoint_path, save_final_checkpoint=False,
            output_path=None, save_mse_every_n_steps=0, save_timing_every_n_steps=0, save_memory_every_n_steps=0,
            synchronize_timing=False, multi_sae_backward_order="forward", multi_sae_stats_sync_mode="immediate",
            multi_sae_stats_sync_interval=1, total_training_samples=self.training_samples, device=self.device,
            autocast=self.autocast, lr=self.lr, lr_end=self.lr_end, lr_scheduler_name=self.lr_scheduler_name,
            lr_warm_up_steps=self.lr_warm_up_steps, adam_beta1=self.adam_beta1, adam_beta2=self.adam_beta2,
            lr_decay_steps=self.lr_decay_steps, n_restart_cycles=1,
            train_batch_size_samples=self.train_batch_size_samples, dead_feature_window=self.dead_feature_window,
            feature_sampling_window=self.feature_sampling_window, logger=self.logger)


@dataclass
class SyntheticSAERunnerResult:
    sae: Any
    synthetic_model: SyntheticModel
    eval_result: SyntheticDataEvalResult
    output_path: Path | None = None


class SyntheticSAERunner:
    def __init__(self, cfg: SyntheticSAERunnerConfig, override_synthetic_model: SyntheticModel | None = None,
                 override_sae: Any = None):
        from saelens_b200.registry import get_sae_training_class

        self.cfg = cfg
        torch.manual_seed(cfg.seed)
        if override_synthetic_model is not None:
            self.model = override_synthetic_model
        elif isinstance(cfg.synthetic_model, SyntheticModelConfig):
            self.model = SyntheticModel(cfg.synthetic_model, device=cfg.device)
        elif isinstance(cfg.synthetic_model, str):
            self.model = SyntheticModel.load_from_source(cfg.synthetic_model, device=cfg.device)
        else:
            raise ValueError("set synthetic_model (config, local path or hub id) or pass override_synthetic_model")
        if override_sae is not None:
            self.sae = override_sae
        else:
            sae_cls, _ = get_sae_training_class(cfg.sae.architecture())
            cfg.sae.device = cfg.device
            self.sae = sae_cls(cfg.sae)
        if self.sae.cfg.d_in != self.model.cfg.hidden_dim:
            raise ValueError(f"SAE d_in {self.sae.cfg.d_in} != synthetic hidden_dim {self.model.cfg.hidden_dim}")

    def run(self) -> SyntheticSAERunnerResult:
        from saelens_b200.training.sae_trainer import SAETrainer

        data = SyntheticActivationIterator(self.model, self.cfg.train_batch_size_samples, dtype=self.sae.W_enc.dtype,
                                           device=self.cfg.device)
        trainer = SAETrainer(self.cfg.to_sae_trainer_config(), self.sae, data)
        trainer.fit()
        self.sae.eval()
        result = eval_sae_on_synthetic_data(self.sae, self.model.feature_dict, self.model.activation_generator,
                                            num_samples=self.cfg.eval_samples,
                                            batch_size=self.cfg.train_batch_size_samples)
        out = None
        if self.cfg.output_path:
            out = Path(self.cfg.output_path)
            out.mkdir(parents=True, exist_ok=True)
            self.sae.save_model(str(out / "sae"))
            (out / RUNNER_CONFIG_FILENAME).write_text(json.dumps(self.cfg.to_dict(), indent=2, default=str))
            (out / "eval_results.json").write_text(json.dumps(result.to_dict(), indent=2))
        return SyntheticSAERunnerResult(self.sae, self.model, result, out)


# ------------------------------------------------------------------------------ plotting helpers
def find_best_feature_ordering(sae_features: torch.Tensor, true_features: torch.Tensor) -> torch.Tensor:
    """Order of the SAE latents by the index of their best-matching true feature (largest |cos|),
    so a similarity plot of the reordered latents runs along the diagonal
    (sae_lens/synthetic/plotting.py:23-43); ties keep the latents' own order."""
    best = cosine_similarities(sae_features.float(), true_features.float()).abs().argmax(dim=1)
    return torch.argsort(best, stable=True)


def find_best_feature_ordering_from_sae(sae: Any, feature_dict: Any) -> torch.Tensor:
    return find_best_feature_ordering(sae.W_dec.detach(), feature_dict.feature_vectors.detach())


def find_best_feature_ordering_across_saes(saes: Iterable[Any], feature_dict: Any) -> torch.Tensor:
    """One ordering for several SAEs (training snapshots): each SAE's own best ordering, scored by
    the mean cosine (to two decimals) along the diagonal it produces; the best-scoring one wins."""
    true = feature_dict.feature_vectors.detach().float()
    best_score, best_order = float("-inf"), None
    for sae in saes:
        w = sae.W_dec.detach().float()
        order = find_best_feature_ordering(w, true)
        sims = torch.round(cosine_similarities(w[order], true) * 100) / 100
        m = min(sims.shape)
        score = float(sims[torch.arange(m), torch.arange(m)].mean())
        if score > best_score:
            best_score, best_order = score, order
    if best_order is None:
        raise ValueError("no SAEs given")
    return best_order


def plot_sae_feature_similarity(sae: Any, feature_dict: Any, reorder_features: bool = True,
                                title: str | None = None, save_path: str | None = None) -> Any:
    """Heatmap of |cos(SAE decoder, ground truth)| (requires matplotlib); returns the figure."""
    import matplotlib

    matplotlib.use("Agg")
    import matplotlib.pyplot as plt

    W = sae.W_dec.detach().float()
    if reorder_features:
        W = W[find_best_feature_ordering_from_sae(sae, feature_dict)]
    sim = cosine_similarities(W, feature_dict.feature_vectors.detach().float()).abs().cpu().numpy()
    fig, ax = plt.subplots(figsize=(6, 5))
    im = ax.imshow(sim, vmin=0, vmax=1, cmap="viridis", aspect="auto")
    ax.set_xlabel("ground-truth feature")
    ax.set_ylabel("SAE latent")
    ax.set_title(title or "SAE decoder vs ground-truth features (|cos|)")
    fig.colorbar(im, ax=ax)
    if save_path:
        fig.savefig(save_path, bbox_inches="tight")
    return fig


def upload_synthetic_model_to_huggingface(model: SyntheticModel | str | Path, repo_id: str,
                                          subfolder: str | None = None, private: bool = False,
                                          revision: str | None = None) -> None:
    """Save (if needed) and upload a synthetic model folder to the Hugging Face hub."""
    import tempfile

    from huggingface_hub import HfApi

    api = HfApi()
    api.create_repo(repo_id, private=private, exist_ok=True)
    with tempfile.TemporaryDirectory() as tmp:
        path = Path(model) if not isinstance(model, SyntheticModel) else Path(tmp) / "model"
        if isinstance(model, SyntheticModel):
            model.save(path)
        api.upload_folder(folder_path=str(path), repo_id=repo_id, path_in_repo=subfolder or ".", revision=revision)
