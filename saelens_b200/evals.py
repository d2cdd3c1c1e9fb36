"""SAE evaluation (metric names and grouping of sae_lens/evals.py).

`run_evals(sae, activation_store, model, eval_config)` returns
(metrics grouped as model_behavior_preservation / model_performance_preservation /
reconstruction_quality / shrinkage / sparsity / token_stats, feature-wise metrics):
* CE loss and KL divergence of the model's next-token predictions with the SAE spliced in,
  against the clean model and against zero-ablating the hook (`ce_loss_score`, `kl_div_score`);
* L0 / L1 of the features, explained variance (pooled and per-token "legacy"), MSE, cosine
  similarity, L2 norms in / out, their ratio and the relative reconstruction bias;
* feature density and a consistent-activation heuristic per latent; encoder/decoder weight
  statistics.
`LLMSaeEvaluator` is the training-time evaluator the runner hands to SAETrainer.
"""

from __future__ import annotations

import argparse
import json
from dataclasses import asdict, dataclass, field
from typing import Any

import torch

from saelens_b200 import __version__


@dataclass
class EvalConfig:
    batch_size_prompts: int | None = None
    n_eval_reconstruction_batches: int = 10
    compute_kl: bool = False
    compute_ce_loss: bool = False
    n_eval_sparsity_variance_batches: int = 1
    compute_l2_norms: bool = False
    compute_sparsity_metrics: bool = False
    compute_variance_metrics: bool = False
    compute_featurewise_density_statistics: bool = False
    compute_featurewise_weight_based_metrics: bool = False
    library_version: str = field(default_factory=lambda: __version__)
    git_hash: str = "unknown"


def get_eval_everything_config(batch_size_prompts: int | None = None, n_eval_reconstruction_batches: int = 10,
                               n_eval_sparsity_variance_batches: int = 1) -> EvalConfig:
    return EvalConfig(batch_size_prompts=batch_size_prompts, n_eval_reconstruction_batches=n_eval_reconstruction_batches,
                      compute_kl=True, compute_ce_loss=True, compute_l2_norms=True,
                      n_eval_sparsity_variance_batches=n_eval_sparsity_variance_batches, compute_sparsity_metrics=True,
                      compute_variance_metrics=True, compute_featurewise_density_statistics=True,
                      compute_featurewise_weight_based_metrics=True)


def _hook_name(sae: Any, store: Any) -> str:
    return sae.cfg.metadata.hook_name or store.hook_name


def _replace_hook(sae: Any, head: int | None, mode: str):
    def hook(act: torch.Tensor, hook: Any) -> torch.Tensor:
        if mode == "zero":
            if head is not None:
                out = act.clone()
                out[:, :, head] = 0
                return out
            return torch.zeros_like(act)
        x = act[:, :, head] if head is not None else act
        shape = x.shape
        flat = x.reshape(-1, shape[-1]) if not getattr(sae, "hook_z_reshaping_mode", False) else x
        rec = sae.decode(sae.encode(flat.to(sae.W_dec.dtype))).to(act.dtype).reshape(shape)
        if head is not None:
            out = act.clone()
            out[:, :, head] = rec
            return out
        return rec
    return hook


@torch.no_grad()
def get_downstream_reconstruction_metrics(sae: Any, model: Any, store: Any, cfg: EvalConfig) -> dict[str, float]:
    hook = _hook_name(sae, store)
    head = store.hook_head_index
    vals: dict[str, list[torch.Tensor]] = {k: [] for k in ("kl_div_with_sae", "kl_div_with_ablation", "ce_loss_with_sae",
                                                            "ce_loss_without_sae", "ce_loss_with_ablation")}
    for _ in range(cfg.n_eval_reconstruction_batches):
        toks = store.get_batch_tokens(cfg.batch_size_prompts)
        dev = getattr(model, "device", None) or next(model.parameters()).device
        toks = toks.to(dev)
        clean = model(toks).float()
        with_sae = model.run_with_hooks(toks, fwd_hooks=[(hook, _replace_hook(sae, head, "sae"))]).float()
        ablated = model.run_with_hooks(toks, fwd_hooks=[(hook, _replace_hook(sae, head, "zero"))]).float()
        lp_clean = torch.log_softmax(clean, -1)

        def kl(other: torch.Tensor) -> torch.Tensor:
            lp = torch.log_softmax(other, -1)
            return (lp_clean.exp() * (lp_clean - lp)).sum(-1).mean(-1)

        def ce(logits: torch.Tensor) -> torch.Tensor:
            lp = torch.log_softmax(logits, -1)[:, :-1]
            return -lp.gather(-1, toks[:, 1:].unsqueeze(-1)).squeeze(-1).mean(-1)

        if cfg.compute_kl:
            vals["kl_div_with_sae"].append(kl(with_sae))
            vals["kl_div_with_ablation"].append(kl(ablated))
        if cfg.compute_ce_loss:
            vals["ce_loss_with_sae"].append(ce(with_sae))
            vals["ce_loss_without_sae"].append(ce(clean))
            vals["ce_loss_with_ablation"].append(ce(ablated))
    m = {k: torch.cat(v).mean().item() for k, v in vals.items() if v}
    if cfg.compute_kl:
        m["kl_div_score"] = (m["kl_div_with_ablation"] - m["kl_div_with_sae"]) / m["kl_div_with_ablation"]
    if cfg.compute_ce_loss:
        denom = m["ce_loss_with_ablation"] - m["ce_loss_without_sae"]
        m["ce_loss_score"] = (m["ce_loss_with_ablation"] - m["ce_loss_with_sae"]) / denom if denom != 0 else float("nan")
    return m


@torch.no_grad()
def get_sparsity_and_variance_metrics(sae: Any, model: Any, store: Any, cfg: EvalConfig) -> tuple[dict[str, float], dict[str, list[float]]]:
    per: dict[str, list[torch.Tensor]] = {k: [] for k in ("l2_norm_in", "l2_norm_out", "l2_ratio", "l0", "l1",
                                                           "explained_variance_legacy", "mse", "cossim")}
    bias_num, bias_den = 0.0, 0.0
    resid_sum, tot_sum = 0.0, 0.0
    feat_sum = torch.zeros(sae.cfg.d_sae)
    feat_tok_active: list[torch.Tensor] = []
    n_tok = 0
    for _ in range(cfg.n_eval_sparsity_variance_batches):
        toks = store.get_batch_tokens(cfg.batch_size_prompts)
        acts = store.get_activations(toks)
        acts = next(iter(acts.values())) if isinstance(acts, dict) else acts
        x = acts.reshape(-1, acts.shape[-1]).to(sae.W_dec.device, sae.W_dec.dtype)
        f = sae.encode(x)
        xh = sae.decode(f)
        x32, xh32, f32 = x.float(), xh.float(), f.float()
        per["l2_norm_in"].append(x32.norm(dim=-1))
        per["l2_norm_out"].append(xh32.norm(dim=-1))
        per["l2_ratio"].append(xh32.norm(dim=-1) / x32.norm(dim=-1).clamp(min=1e-12))
        bias_num += (xh32 * x32).sum().item()
        bias_den += x32.pow(2).sum().item()
        per["l0"].append((f32 > 0).float().sum(-1))
        per["l1"].append(f32.abs().sum(-1))
        r2 = (x32 - xh32).pow(2).sum(-1)
        tv = (x32 - x32.mean(0)).pow(2).sum(-1)
        per["explained_variance_legacy"].append(1 - r2 / tv.clamp(min=1e-12))
        resid_sum += r2.sum().item()
        tot_sum += tv.sum().item()
        per["mse"].append(r2 / x.shape[-1])
        per["cossim"].append(torch.nn.functional.cosine_similarity(x32, xh32, dim=-1))
        feat_sum += (f32 > 0).float().sum(0).cpu()
        feat_tok_active.append(f32.cpu())
        n_tok += x.shape[0]
    m = {k: torch.cat(v).mean().item() for k, v in per.items()}
    m["relative_reconstruction_bias"] = bias_num / bias_den if bias_den else float("nan")
    m["explained_variance"] = 1 - resid_sum / tot_sum if tot_sum else float("nan")
    fm: dict[str, list[float]] = {}
    if cfg.compute_featurewise_density_statistics:
        allf = torch.cat(feat_tok_active)
        fm["feature_density"] = (feat_sum / max(n_tok, 1)).tolist()
        fired = allf > 0
        mean_when = (allf * fired).sum(0) / fired.sum(0).clamp(min=1)
        fm["consistent_activation_heuristic"] = (mean_when / allf.max(0).values.clamp(min=1e-12)).tolist()
    return m, fm


@torch.no_grad()
def get_featurewise_weight_based_metrics(sae: Any) -> dict[str, list[float]]:
    We = sae.W_enc.detach().float()
    Wd = sae.W_dec.detach().float()
    out = {"encoder_norm": We.norm(dim=0).tolist(),
           "encoder_decoder_cosine_sim": torch.nn.functional.cosine_similarity(We.T, Wd, dim=-1).tolist()}
    if hasattr(sae, "b_enc"):
        out["encoder_bias"] = sae.b_enc.detach().float().cpu().tolist()
    return out


@torch.no_grad()
def run_evals(sae: Any, activation_store: Any, model: Any, eval_config: EvalConfig = EvalConfig(),
              model_kwargs: dict[str, Any] | None = None, ignore_tokens: set[int | None] | None = None,
              verbose: bool = False) -> tuple[dict[str, Any], dict[str, Any]]:
    del model_kwargs, ignore_tokens, verbose
    metrics: dict[str, Any] = {k: {} for k in ("model_behavior_preservation", "model_performance_preservation",
                                               "reconstruction_quality", "shrinkage", "sparsity", "token_stats")}
    feat: dict[str, Any] = {}
    bs = eval_config.batch_size_prompts or activation_store.store_batch_size_prompts
    ctx = activation_store.context_size
    if eval_config.compute_kl or eval_config.compute_ce_loss:
        r = get_downstream_reconstruction_metrics(sae, model, activation_store, eval_config)
        if eval_config.compute_kl:
            metrics["model_behavior_preservation"].update(
                {k: r[k] for k in ("kl_div_score", "kl_div_with_ablation", "kl_div_with_sae")})
        if eval_config.compute_ce_loss:
            metrics["model_performance_preservation"].update(
                {k: r[k] for k in ("ce_loss_score", "ce_loss_with_ablation", "ce_loss_with_sae", "ce_loss_without_sae")})
    if (eval_config.compute_l2_norms or eval_config.compute_sparsity_metrics or eval_config.compute_variance_metrics
            or eval_config.compute_featurewise_density_statistics):
        m, fm = get_sparsity_and_variance_metrics(sae, model, activation_store, eval_config)
        if eval_config.compute_l2_norms:
            metrics["shrinkage"].update({k: m[k] for k in ("l2_norm_in", "l2_norm_out", "l2_ratio",
                                                           "relative_reconstruction_bias")})
        if eval_config.compute_sparsity_metrics:
            metrics["sparsity"].update({"l0": m["l0"], "l1": m["l1"]})
        if eval_config.compute_variance_metrics:
            metrics["reconstruction_quality"].update({k: m[k] for k in ("explained_variance", "explained_variance_legacy",
                                                                        "mse", "cossim")})
        feat.update(fm)
    if eval_config.compute_featurewise_weight_based_metrics:
        feat.update(get_featurewise_weight_based_metrics(sae))
    metrics["token_stats"] = {
        "total_tokens_eval_reconstruction": eval_config.n_eval_reconstruction_batches * bs * ctx
        if (eval_config.compute_kl or eval_config.compute_ce_loss) else 0,
        "total_tokens_eval_sparsity_variance": eval_config.n_eval_sparsity_variance_batches * bs * ctx,
    }
    metrics = {k: v for k, v in metrics.items() if v}
    return metrics, feat


class LLMSaeEvaluator:
    """Evaluator used during training: reconstruction CE/KL plus sparsity / variance metrics."""

    def __init__(self, model: Any, store: Any, n_eval_batches: int, eval_batch_size_prompts: int | None):
        self.model, self.store = model, store
        self.cfg = EvalConfig(batch_size_prompts=eval_batch_size_prompts, n_eval_reconstruction_batches=n_eval_batches,
                              compute_kl=True, compute_ce_loss=True, compute_l2_norms=True,
                              compute_sparsity_metrics=True, compute_variance_metrics=True)

    def __call__(self, sae: Any, data_provider: Any, activation_scaler: Any) -> dict[str, Any]:
        del data_provider, activation_scaler
        metrics, _ = run_evals(sae, self.store, self.model, self.cfg)
        return {f"eval/{g}/{k}": v for g, d in metrics.items() for k, v in d.items()}


def process_results(eval_results: list[dict[str, Any]], output_dir: str) -> dict[str, str]:
    from pathlib import Path

    out = Path(output_dir)
    out.mkdir(parents=True, exist_ok=True)
    p = out / "eval_results.json"
    p.write_text(json.dumps(eval_results, indent=2))
    return {"json": str(p)}


def run_evals_cli(argv: list[str] | None = None) -> None:
    """`python -m saelens_b200.evals <sae_path> --model <preset> --dataset <src> --output-dir <dir>`."""
    ap = argparse.ArgumentParser()
    ap.add_argument("sae_path")
    ap.add_argument("--model", required=True)
    ap.add_argument("--dataset", required=True)
    ap.add_argument("--output-dir", default="eval_results")
    ap.add_argument("--batch-size-prompts", type=int, default=8)
    ap.add_argument("--n-batches", type=int, default=2)
    ap.add_argument("--device", default="cuda" if torch.cuda.is_available() else "cpu")
    a = ap.parse_args(argv)
    from saelens_b200.models.lm.load_model import load_model
    from saelens_b200.models.sae import SAE
    from saelens_b200.training.activations_store import ActivationsStore

    sae = SAE.load_from_disk(a.sae_path, device=a.device)
    model = load_model("HookedTransformer", a.model, device=a.device)
    store = ActivationsStore.from_sae(model, sae, a.dataset, store_batch_size_prompts=a.batch_size_prompts,
                                      device=a.device)
    cfg = get_eval_everything_config(a.batch_size_prompts, a.n_batches, a.n_batches)
    metrics, feat = run_evals(sae, store, model, cfg)
    process_results([{"sae_path": a.sae_path, "metrics": metrics, "eval_config": asdict(cfg)}], a.output_dir)


if __name__ == "__main__":
    run_evals_cli()
