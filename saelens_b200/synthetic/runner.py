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
from saelens_b200.synthetic.model import (
    SYNTHETIC_MODEL_CONFIG_FILENAME,
    SyntheticActivationIterator,
    SyntheticModel,
    SyntheticModelConfig,
)
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


def feature_similarity_matrices(sae: Any, feature_dict: Any,
                                reorder_features: bool | torch.Tensor = False) -> tuple[torch.Tensor, torch.Tensor]:
    """(encoder, decoder) cosine similarities of the SAE latents with the true features, rounded
    to two decimals, rows reordered by `find_best_feature_ordering` (True) or by the given index
    tensor: the matrices `plot_sae_feature_similarity` draws."""
    true = feature_dict.feature_vectors.detach().float()
    dec = torch.round(cosine_similarities(sae.W_dec.detach().float(), true) * 100) / 100
    enc = torch.round(cosine_similarities(sae.W_enc.detach().float().T, true) * 100) / 100
    if reorder_features is not False:
        order = (find_best_feature_ordering(sae.W_dec.detach(), true) if isinstance(reorder_features, bool)
                 else reorder_features)
        dec, enc = dec[order], enc[order]
    return enc, dec


def plot_sae_feature_similarity(sae: Any, feature_dict: Any, title: str | None = None,
                                reorder_features: bool | torch.Tensor = False, decoder_only: bool = False,
                                show_values: bool = False, height: int = 400, width: int = 800,
                                save_path: str | Path | None = None, show_plot: bool = True, dtick: int | None = 1,
                                scale: float = 1.0) -> Any:
    """Heatmaps of the SAE encoder's and decoder's cosine similarity with the true features
    (sae_lens/synthetic/plotting.py:102-230; plotly, an optional dependency as in the reference).
    Returns the figure."""
    try:
        import plotly.graph_objects as go
        from plotly.subplots import make_subplots
    except ImportError as e:  # pragma: no cover - depends on the environment
        raise ImportError("plot_sae_feature_similarity needs plotly (pip install plotly)") from e
    enc, dec = feature_similarity_matrices(sae, feature_dict, reorder_features)
    hover = "True feature: %{x}<br>SAE Latent: %{y}<br>Cosine Similarity: %{z:.3f}<extra></extra>"

    def heatmap(z: torch.Tensor, with_scale: bool) -> Any:
        kw: dict[str, Any] = {"z": z.cpu().numpy(), "zmin": -1, "zmax": 1, "colorscale": "RdBu",
                              "hovertemplate": hover}
        if with_scale:
            kw["colorbar"] = {"title": "cos sim", "x": 1.0, "dtick": 1, "tickvals": [-1, 0, 1]}
        else:
            kw["showscale"] = False
        if show_values:
            kw.update(texttemplate="%{z:.2f}", textfont={"size": 10})
        return go.Heatmap(**kw)

    panels = [("SAE decoder", dec, True)] if decoder_only else [("SAE encoder", enc, False), ("SAE decoder", dec, True)]
    fig = make_subplots(rows=1, cols=len(panels),
                        subplot_titles=None if decoder_only else tuple(name for name, _, _ in panels))
    for col, (_, z, with_scale) in enumerate(panels, start=1):
        fig.add_trace(heatmap(z, with_scale), row=1, col=col)
        fig.update_xaxes(title_text="True feature", row=1, col=col, dtick=dtick)
        fig.update_yaxes(title_text="SAE Latent", row=1, col=col, dtick=dtick)
    fig.update_layout(height=height, width=width, title_text=title or "Cosine similarity with true features")
    if save_path:
        Path(save_path).parent.mkdir(parents=True, exist_ok=True)
        fig.write_image(str(save_path), scale=scale)
    if show_plot:
        fig.show()
    return fig


def upload_synthetic_model_to_huggingface(model: SyntheticModel | str | Path, hf_repo_id: str,
                                          hf_path: str | None = None, hf_revision: str = "main",
                                          add_default_readme: bool = True, private: bool = False) -> None:
    """Save (if given as a model) and upload a synthetic model folder to the Hugging Face hub, at
    the repo root or in `hf_path`; with `add_default_readme` a README.md describing the model is
    added when the repo has none (sae_lens/synthetic/upload_synthetic_model.py:24-71)."""
    import io
    import tempfile

    from huggingface_hub import HfApi

    api = HfApi()
    api.create_repo(hf_repo_id, private=private, exist_ok=True)
    with tempfile.TemporaryDirectory() as tmp:
        path = Path(model) if not isinstance(model, SyntheticModel) else Path(tmp) / "model"
        if isinstance(model, SyntheticModel):
            model.save(path)
        if not (path / SYNTHETIC_MODEL_CONFIG_FILENAME).exists():
            raise FileNotFoundError(f"{path} holds no {SYNTHETIC_MODEL_CONFIG_FILENAME}")
        api.upload_folder(folder_path=str(path), repo_id=hf_repo_id, path_in_repo=hf_path or ".",
                          revision=hf_revision)
        if add_default_readme and not api.file_exists(hf_repo_id, "README.md", revision=hf_revision):
            synth = model if isinstance(model, SyntheticModel) else SyntheticModel.load_from_disk(path)
            text = default_synthetic_model_readme(hf_repo_id, hf_path, synth)
            api.upload_file(path_or_fileobj=io.BytesIO(text.encode("utf-8")), path_in_repo="README.md",
                            repo_id=hf_repo_id, revision=hf_revision, commit_message="Add README.md")


def default_synthetic_model_readme(repo_id: str, path: str | None, model: SyntheticModel) -> str:
    """README of an uploaded synthetic model: its sizes, its generators and how to load it."""
    cfg = model.cfg
    where = f'"{repo_id}", model_path="{path}"' if path else f'"{repo_id}"'
    lines = [
        "---", "library_name: saelens", "tags:", "- synthetic", "- sparse-autoencoder", "---", "",
        f"# Synthetic model `{repo_id}`" + (f" (`{path}`)" if path else ""), "",
        "Ground-truth feature dictionary and activation generator for benchmarking sparse autoencoders.", "",
        f"* features: {cfg.num_features}", f"* hidden dimension: {cfg.hidden_dim}",
        f"* firing probabilities: {cfg.firing_probability.to_dict()}",
        f"* hierarchy: {'yes' if cfg.hierarchy is not None else 'no'}",
        f"* correlation: {'low-rank' if cfg.correlation is not None else 'none'}", "",
        "```python", "from saelens_b200.synthetic import SyntheticModel", "",
        f"model = SyntheticModel.from_pretrained({where})", "hidden = model.sample(1024)", "```", "",
    ]
    return "\n".join(lines)
