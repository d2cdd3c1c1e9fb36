"""SAE evaluation: the metric names, grouping and definitions of sae_lens/evals.py, so numbers are
comparable between the two frameworks.

`run_evals(sae, activation_store, model, activation_scaler, eval_config)` returns
(metrics grouped as model_behavior_preservation / model_performance_preservation /
reconstruction_quality / shrinkage / sparsity / token_stats, feature-wise metrics):

* downstream (sae_lens/evals.py:315-381, 601-755): per-token KL(clean || spliced) and next-token CE
  with the SAE spliced in, without it and with the hook zero-ablated; tokens in the ignore set
  (special tokens by default) keep their clean activation and are left out of the means;
  `kl_div_score = (KL_abl - KL_sae) / KL_abl`, `ce_loss_score = (CE_abl - CE_sae) / (CE_abl - CE_clean)`;
* sparsity / variance over the unmasked tokens (sae_lens/evals.py:384-598): L2 norms in / out and
  their ratio (inputs with norm < 1e-4 divide by 1), relative reconstruction bias
  `mean ||x_hat||^2 / mean <x, x_hat>` per batch, L0, L1 (sum of activations), the legacy
  per-token explained variance, `mse` = per-token residual sum of squares / number of unmasked
  tokens, cosine similarity, and `explained_variance = 1 - E[rss] / (E[||x||^2] - (E[x^2])^2)`
  with E[x^2] averaged over tokens and dimensions;
* feature-wise: density (firings / unmasked tokens), the consistent-activation heuristic
  (firings / prompts with at least one firing), encoder norms, encoder-decoder cosine and b_enc.

Attention hooks (`hook_q/k/v/z`) are evaluated on their flattened heads, or on one head with
`hook_head_index`; an SAE in hook_z reshaping mode is switched out of it for the evaluation and
back afterwards.  `run_evals_cli` evaluates every pretrained SAE whose release and id match two
regular expressions (sae_lens/evals.py:758-1064).
"""

from __future__ import annotations

import argparse
import json
import math
import re
from collections import defaultdict
from collections.abc import Iterable, Mapping
from dataclasses import dataclass, field
from pathlib import Path
from typing import Any

import torch

from saelens_b200 import __version__
from saelens_b200.training.activation_scaler import ActivationScaler
from saelens_b200.utils.misc import extract_stop_at_layer_from_tlens_hook_name, get_special_token_ids

_HEAD_HOOKS = ("hook_q", "hook_k", "hook_v", "hook_z")


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


def _keep_mask(tokens: torch.Tensor, ignore_tokens: list[int] | None) -> torch.Tensor:
    """True where a token is evaluated (not one of `ignore_tokens`)."""
    if not ignore_tokens:
        return torch.ones_like(tokens, dtype=torch.bool)
    return ~torch.isin(tokens, torch.tensor(list(ignore_tokens), dtype=tokens.dtype, device=tokens.device))


def _model_device(model: Any) -> torch.device:
    dev = getattr(model, "device", None)
    return torch.device(dev) if dev is not None else next(model.parameters()).device


def _logits(out: Any) -> torch.Tensor:
    return out.logits if hasattr(out, "logits") else out


def _ce_per_token(logits: torch.Tensor, tokens: torch.Tensor) -> torch.Tensor:
    """[B, S-1] next-token cross entropy."""
    lp = torch.log_softmax(logits.float(), -1)[:, :-1]
    return -lp.gather(-1, tokens[:, 1:].unsqueeze(-1)).squeeze(-1)


def _kl(original_logits: torch.Tensor, new_logits: torch.Tensor) -> torch.Tensor:
    """[B, S] KL(original || new) per token."""
    lp_orig = torch.log_softmax(original_logits.float(), -1)
    lp_new = torch.log_softmax(new_logits.float(), -1)
    return (lp_orig.exp() * (lp_orig - lp_new)).sum(-1)


@torch.no_grad()
def get_recons_loss(sae: Any, model: Any, activation_scaler: ActivationScaler, batch_tokens: torch.Tensor,
                    compute_kl: bool, compute_ce_loss: bool, ignore_tokens: list[int] | None = None,
                    model_kwargs: Mapping[str, Any] | None = None, hook_name: str | None = None) -> dict[str, torch.Tensor]:
    """Per-token KL ([B, S]) and CE ([B, S-1]) of the clean, SAE-spliced and zero-ablated model."""
    hook_name = hook_name or sae.cfg.metadata.hook_name
    if hook_name is None:
        raise ValueError("hook_name must be provided")
    head = sae.cfg.metadata.hook_head_index
    kw = dict(model_kwargs or {})
    keep = _keep_mask(batch_tokens, ignore_tokens)
    head_dim = any(s in hook_name for s in _HEAD_HOOKS)

    def run_sae(a: torch.Tensor) -> torch.Tensor:
        return activation_scaler.unscale(sae.decode(sae.encode(activation_scaler.scale(a.to(sae.W_dec.device)))))

    def replace(acts: torch.Tensor, hook: Any) -> torch.Tensor:
        if head_dim and head is not None:
            out = acts.clone()
            out[:, :, head] = run_sae(acts[:, :, head]).to(acts.dtype).to(acts.device)
            return out
        if head_dim:
            new = run_sae(acts.flatten(-2, -1)).reshape(acts.shape)
        else:
            new = run_sae(acts)
        new = new.to(acts.dtype).to(acts.device)
        m = keep.to(acts.device).reshape(keep.shape + (1,) * (acts.dim() - 2))
        return torch.where(m, new, acts)

    def ablate(acts: torch.Tensor, hook: Any) -> torch.Tensor:
        if head_dim and head is not None:
            out = acts.clone()
            out[:, :, head] = 0
            return out
        return torch.zeros_like(acts)

    toks = batch_tokens.to(_model_device(model))
    clean = _logits(model(toks, **kw))
    spliced = _logits(model.run_with_hooks(toks, fwd_hooks=[(hook_name, replace)], **kw))
    ablated = _logits(model.run_with_hooks(toks, fwd_hooks=[(hook_name, ablate)], **kw))
    out: dict[str, torch.Tensor] = {}
    if compute_kl:
        out["kl_div_with_sae"] = _kl(clean, spliced)
        out["kl_div_with_ablation"] = _kl(clean, ablated)
    if compute_ce_loss:
        out["ce_loss_with_sae"] = _ce_per_token(spliced, toks)
        out["ce_loss_without_sae"] = _ce_per_token(clean, toks)
        out["ce_loss_with_ablation"] = _ce_per_token(ablated, toks)
    return out


@torch.no_grad()
def get_downstream_reconstruction_metrics(sae: Any, model: Any, activation_store: Any,
                                          activation_scaler: ActivationScaler, compute_kl: bool, compute_ce_loss: bool,
                                          n_batches: int, eval_batch_size_prompts: int,
                                          ignore_tokens: list[int] | None = None, verbose: bool = False,
                                          model_kwargs: Mapping[str, Any] | None = None) -> dict[str, float]:
    del verbose
    vals: dict[str, list[torch.Tensor]] = defaultdict(list)
    for _ in range(n_batches):
        toks = activation_store.get_batch_tokens(eval_batch_size_prompts)
        keep = _keep_mask(toks, ignore_tokens)
        for name, v in get_recons_loss(sae, model, activation_scaler, toks, compute_kl, compute_ce_loss,
                                       ignore_tokens, model_kwargs).items():
            if ignore_tokens:
                m = keep if v.shape[1] == keep.shape[1] else keep[:, :-1]  # CE has no last position
                v = v[m.to(v.device)]
            vals[name].append(v.flatten())
    m: dict[str, float] = {k: torch.cat(v).mean().item() for k, v in vals.items()}
    if compute_kl:
        m["kl_div_score"] = (m["kl_div_with_ablation"] - m["kl_div_with_sae"]) / m["kl_div_with_ablation"]
    if compute_ce_loss:
        denom = m["ce_loss_with_ablation"] - m["ce_loss_without_sae"]
        m["ce_loss_score"] = (m["ce_loss_with_ablation"] - m["ce_loss_with_sae"]) / denom if denom else float("nan")
    return m


@torch.no_grad()
def get_sparsity_and_variance_metrics(sae: Any, model: Any, activation_store: Any, activation_scaler: ActivationScaler,
                                      n_batches: int, compute_l2_norms: bool, compute_sparsity_metrics: bool,
                                      compute_variance_metrics: bool, compute_featurewise_density_statistics: bool,
                                      eval_batch_size_prompts: int, model_kwargs: Mapping[str, Any] | None = None,
                                      ignore_tokens: list[int] | None = None,
                                      verbose: bool = False) -> tuple[dict[str, float], dict[str, list[float]]]:
    del verbose
    hook_name = sae.cfg.metadata.hook_name
    head = sae.cfg.metadata.hook_head_index
    per: dict[str, list[torch.Tensor]] = defaultdict(list)
    sumsq, act_sq, rss_means = [], [], []
    d_sae = sae.cfg.d_sae
    fires = torch.zeros(d_sae)
    prompts_fired = torch.zeros(d_sae)
    n_tokens = 0
    for _ in range(n_batches):
        toks = activation_store.get_batch_tokens(eval_batch_size_prompts)
        keep = _keep_mask(toks, ignore_tokens)
        _, cache = model.run_with_cache(toks.to(_model_device(model)), names_filter=[hook_name],
                                        stop_at_layer=extract_stop_at_layer_from_tlens_hook_name(hook_name),
                                        **dict(model_kwargs or {}))
        act = cache[hook_name]
        if head is not None:
            act = act[:, :, head]
        elif any(s in hook_name for s in _HEAD_HOOKS):
            act = act.flatten(-2, -1)
        x = act.to(sae.W_dec.device, sae.W_dec.dtype)
        f = sae.encode(activation_scaler.scale(x))
        x_hat = activation_scaler.unscale(sae.decode(f))
        if f.is_sparse:
            f = f.to_dense()
        keep_flat = keep.flatten().to(x.device)
        xi = x.reshape(-1, x.shape[-1])[keep_flat].float()
        xo = x_hat.reshape(-1, x_hat.shape[-1])[keep_flat].float()
        fa = f.reshape(-1, f.shape[-1])[keep_flat].float()
        if compute_l2_norms:
            n_in, n_out = xi.norm(dim=-1), xo.norm(dim=-1)
            div = torch.where(n_in.abs() < 1e-4, torch.ones_like(n_in), n_in)
            per["l2_norm_in"].append(n_in)
            per["l2_norm_out"].append(n_out)
            per["l2_ratio"].append(n_out / div)
            per["relative_reconstruction_bias"].append(((n_out ** 2).mean() / (xi * xo).sum(-1).mean()).reshape(1))
        if compute_sparsity_metrics:
            per["l0"].append((fa > 0).sum(-1).float())
            per["l1"].append(fa.sum(-1))
        if compute_variance_metrics:
            rss = (xi - xo).pow(2).sum(-1)
            per["mse"].append(rss / keep_flat.sum())
            per["explained_variance_legacy"].append(1 - rss / (xi - xi.mean(0)).pow(2).sum(-1))
            sumsq.append(xi.pow(2).sum(-1).mean(0))
            act_sq.append(xi.pow(2).mean(0))
            rss_means.append(rss.mean(0))
            per["cossim"].append((xi / xi.norm(dim=-1, keepdim=True) * (xo / xo.norm(dim=-1, keepdim=True))).sum(-1))
        if compute_featurewise_density_statistics:
            fired = ((f.float() * keep.to(f.device).unsqueeze(-1)) > 0).float()
            fires += fired.sum(dim=1).sum(dim=0).cpu()
            prompts_fired += (fired.sum(dim=1) > 0).sum(dim=0).float().cpu()
            n_tokens += int(keep.sum())
    metrics = {k: torch.cat(v).mean().item() for k, v in per.items()}
    if compute_variance_metrics:
        total_var = torch.stack(sumsq).mean(0) - torch.cat(act_sq).mean(0) ** 2
        metrics["explained_variance"] = (1 - torch.stack(rss_means).mean(0) / total_var).item()
    feature: dict[str, list[float]] = {}
    if compute_featurewise_density_statistics:
        feature["feature_density"] = (fires / max(n_tokens, 1)).tolist()
        feature["consistent_activation_heuristic"] = (fires / prompts_fired).tolist()
    return metrics, feature


@torch.no_grad()
def get_featurewise_weight_based_metrics(sae: Any) -> dict[str, Any]:
    We = sae.W_enc.detach().float().cpu()
    Wd = sae.W_dec.detach().float().cpu()
    out: dict[str, Any] = {
        "encoder_norm": We.norm(dim=-2).tolist(),
        "encoder_decoder_cosine_sim": torch.nn.functional.cosine_similarity(Wd / Wd.norm(dim=-1, keepdim=True),
                                                                            (We / We.norm(dim=0, keepdim=True)).T).tolist(),
    }
    if getattr(sae, "b_enc", None) is not None:
        out["encoder_bias"] = sae.b_enc.detach().float().cpu().tolist()
    return out


@torch.no_grad()
def run_evals(sae: Any, activation_store: Any, model: Any, activation_scaler: ActivationScaler | None = None,
              eval_config: EvalConfig = EvalConfig(), model_kwargs: Mapping[str, Any] | None = None,
              exclude_special_tokens: Iterable[int] | bool = True,
              verbose: bool = False) -> tuple[dict[str, Any], dict[str, Any]]:
    """`exclude_special_tokens`: True = the model tokenizer's special ids (none without a
    tokenizer), an iterable = those ids, False = evaluate every token."""
    if isinstance(activation_scaler, EvalConfig):  # (sae, store, model, eval_config) call form
        activation_scaler, eval_config = None, activation_scaler
    scaler = activation_scaler if activation_scaler is not None else ActivationScaler()
    ignore: list[int] | None = None
    if exclude_special_tokens is True:
        tok = getattr(model, "tokenizer", None)
        ignore = list(get_special_token_ids(tok)) if tok is not None else None
    elif exclude_special_tokens:
        ignore = list(exclude_special_tokens)
    hook_name = sae.cfg.metadata.hook_name or activation_store.hook_name
    if sae.cfg.metadata.hook_name is None:
        sae.cfg.metadata.hook_name = hook_name
    prev_z = getattr(sae, "hook_z_reshaping_mode", None) if "hook_z" in hook_name else None
    if prev_z:
        sae.turn_off_forward_pass_hook_z_reshaping()
    bs = eval_config.batch_size_prompts or activation_store.store_batch_size_prompts
    metrics: dict[str, Any] = {k: {} for k in ("model_behavior_preservation", "model_performance_preservation",
                                               "reconstruction_quality", "shrinkage", "sparsity", "token_stats")}
    feature: dict[str, Any] = {}
    try:
        if eval_config.compute_kl or eval_config.compute_ce_loss:
            if eval_config.n_eval_reconstruction_batches <= 0:
                raise ValueError("eval_config.n_eval_reconstruction_batches must be > 0 when "
                                 "compute_kl or compute_ce_loss is True.")
            r = get_downstream_reconstruction_metrics(sae, model, activation_store, scaler, eval_config.compute_kl,
                                                      eval_config.compute_ce_loss,
                                                      eval_config.n_eval_reconstruction_batches, bs, ignore, verbose,
                                                      model_kwargs)
            if eval_config.compute_kl:
                metrics["model_behavior_preservation"].update(
                    {k: r[k] for k in ("kl_div_score", "kl_div_with_ablation", "kl_div_with_sae")})
            if eval_config.compute_ce_loss:
                metrics["model_performance_preservation"].update(
                    {k: r[k] for k in ("ce_loss_score", "ce_loss_with_ablation", "ce_loss_with_sae",
                                       "ce_loss_without_sae")})
            activation_store.reset_input_dataset()
        if eval_config.compute_l2_norms or eval_config.compute_sparsity_metrics or eval_config.compute_variance_metrics:
            if eval_config.n_eval_sparsity_variance_batches <= 0:
                raise ValueError("eval_config.n_eval_sparsity_variance_batches must be > 0 when compute_l2_norms, "
                                 "compute_sparsity_metrics, or compute_variance_metrics is True.")
            m, feature = get_sparsity_and_variance_metrics(
                sae, model, activation_store, scaler, eval_config.n_eval_sparsity_variance_batches,
                eval_config.compute_l2_norms, eval_config.compute_sparsity_metrics,
                eval_config.compute_variance_metrics, eval_config.compute_featurewise_density_statistics, bs,
                model_kwargs, ignore, verbose)
            if eval_config.compute_l2_norms:
                metrics["shrinkage"].update({k: m[k] for k in ("l2_norm_in", "l2_norm_out", "l2_ratio",
                                                               "relative_reconstruction_bias")})
            if eval_config.compute_sparsity_metrics:
                metrics["sparsity"].update({"l0": m["l0"], "l1": m["l1"]})
            if eval_config.compute_variance_metrics:
                metrics["reconstruction_quality"].update(
                    {k: m[k] for k in ("explained_variance", "explained_variance_legacy", "mse", "cossim")})
        if eval_config.compute_featurewise_weight_based_metrics:
            feature |= get_featurewise_weight_based_metrics(sae)
    finally:
        if prev_z:
            sae.turn_on_forward_pass_hook_z_reshaping()
    ctx = activation_store.context_size
    metrics["token_stats"] = {
        "total_tokens_eval_reconstruction": ctx * eval_config.n_eval_reconstruction_batches * bs,
        "total_tokens_eval_sparsity_variance": ctx * eval_config.n_eval_sparsity_variance_batches * bs,
    }
    return {k: v for k, v in metrics.items() if v}, feature


class LLMSaeEvaluator:
    """Evaluator used during training: reconstruction CE/KL plus sparsity / variance metrics."""

    def __init__(self, model: Any, store: Any, n_eval_batches: int, eval_batch_size_prompts: int | None):
        self.model, self.store = model, store
        self.cfg = EvalConfig(batch_size_prompts=eval_batch_size_prompts, n_eval_reconstruction_batches=n_eval_batches,
                              compute_kl=True, compute_ce_loss=True, compute_l2_norms=True,
                              compute_sparsity_metrics=True, compute_variance_metrics=True)

    def __call__(self, sae: Any, data_provider: Any, activation_scaler: Any) -> dict[str, Any]:
        """Evaluates on the training store's tokens and then puts its token position back, so the
        training stream continues where it was."""
        del data_provider
        pos = self.store.token_position() if hasattr(self.store, "token_position") else None
        if pos is not None:  # evaluate on a separate token reader; the training one stays untouched
            self.store.restore_token_position((pos[0], None))
        try:
            metrics, _ = run_evals(sae, self.store, self.model, activation_scaler=activation_scaler,
                                   eval_config=self.cfg)
        finally:
            if pos is not None:
                self.store.restore_token_position(pos)
        return {f"eval/{g}/{k}": v for g, d in metrics.items() for k, v in d.items()}


# ---------------------------------------------------------------------------------------- CLI
def all_loadable_saes() -> list[tuple[str, str, float, float]]:
    """(release, sae id, expected variance explained, expected L0) of every directory entry."""
    from saelens_b200.loading.pretrained_saes_directory import get_pretrained_saes_directory

    out = []
    for release, lookup in get_pretrained_saes_directory().items():
        for sae_id in lookup.saes_map:
            out.append((release, sae_id, lookup.expected_var_explained.get(sae_id),
                        lookup.expected_l0.get(sae_id)))
    return out


def get_saes_from_regex(sae_regex_pattern: str, sae_block_pattern: str) -> list[tuple[str, str, float, float]]:
    rel, blk = re.compile(sae_regex_pattern), re.compile(sae_block_pattern)
    return [s for s in all_loadable_saes() if rel.fullmatch(s[0]) and blk.fullmatch(s[1])]


def nested_dict() -> defaultdict[Any, Any]:
    return defaultdict(nested_dict)


def multiple_evals(sae_regex_pattern: str, sae_block_pattern: str, n_eval_reconstruction_batches: int,
                   n_eval_sparsity_variance_batches: int, eval_batch_size_prompts: int = 8,
                   datasets: list[str] | None = None, dataset_trust_remote_code: bool = False,
                   ctx_lens: list[int] | None = None, output_dir: str = "eval_results",
                   verbose: bool = False) -> list[dict[str, Any]]:
    from saelens_b200.models.lm.load_model import load_model
    from saelens_b200.models.sae import SAE
    from saelens_b200.training.activations_store import ActivationsStore

    del dataset_trust_remote_code
    datasets = datasets or ["Skylion007/openwebtext", "lighteval/MATH"]
    ctx_lens = ctx_lens or [128]
    device = "cuda" if torch.cuda.is_available() else "cpu"
    chosen = get_saes_from_regex(sae_regex_pattern, sae_block_pattern)
    if not chosen:
        raise ValueError("No SAEs matched the given regex patterns")
    Path(output_dir).mkdir(parents=True, exist_ok=True)
    cfg = get_eval_everything_config(eval_batch_size_prompts, n_eval_reconstruction_batches,
                                     n_eval_sparsity_variance_batches)
    results: list[dict[str, Any]] = []
    model, model_name = None, None
    for release, sae_id, _, _ in chosen:
        sae = SAE.from_pretrained(release=release, sae_id=sae_id, device=device)
        if model_name != sae.cfg.metadata.model_name:
            model_name = sae.cfg.metadata.model_name
            model = load_model("HookedTransformer", model_name, device=device,
                               model_from_pretrained_kwargs=sae.cfg.metadata.model_from_pretrained_kwargs or {})
        for ctx in ctx_lens:
            for ds in datasets:
                store = ActivationsStore.from_sae(model, sae, ds, context_size=ctx, device=device)
                store.shuffle_input_dataset(seed=42)
                r = nested_dict()
                r["unique_id"] = f"{release}-{sae_id}"
                r["sae_set"] = release
                r["sae_id"] = sae_id
                r["eval_cfg"]["context_size"] = ctx
                r["eval_cfg"]["dataset"] = ds
                scalar, feat = run_evals(sae, store, model, ActivationScaler(), cfg, verbose=verbose)
                r["metrics"] = scalar
                r["feature_metrics"] = feat
                r["sae_cfg"] = sae.cfg.to_dict()
                r["eval_cfg"].update(cfg.__dict__)
                results.append(r)
    return results


def run_evaluations(args: argparse.Namespace) -> list[dict[str, Any]]:
    chosen = get_saes_from_regex(args.sae_regex_pattern, args.sae_block_pattern)
    print("Filtered SAEs based on provided patterns:")
    print(f"Number of SAE sets: {len({s[0] for s in chosen})}")
    print(f"Total number of SAE IDs: {len(chosen)}")
    return multiple_evals(args.sae_regex_pattern, args.sae_block_pattern, args.n_eval_reconstruction_batches,
                          args.n_eval_sparsity_variance_batches, args.batch_size_prompts, args.datasets,
                          args.dataset_trust_remote_code, args.ctx_lens, args.output_dir, args.verbose)


def replace_nans_with_negative_one(obj: Any) -> Any:
    if isinstance(obj, dict):
        return {k: replace_nans_with_negative_one(v) for k, v in obj.items()}
    if isinstance(obj, list):
        return [replace_nans_with_negative_one(v) for v in obj]
    if isinstance(obj, float) and math.isnan(obj):
        return -1
    return obj


def process_results(eval_results: list[dict[str, Any]], output_dir: str) -> dict[str, Any]:
    """One JSON per result (`<unique_id>_<context>_<dataset>.json`), all results in
    `all_eval_results.json` and a flattened `all_eval_results.csv`; NaNs are written as -1."""
    out = Path(output_dir)
    out.mkdir(parents=True, exist_ok=True)
    cleaned = [replace_nans_with_negative_one(r) for r in eval_results]
    for r in cleaned:
        cfg = r.get("eval_cfg", {})
        name = f"{r['unique_id']}_{cfg.get('context_size')}_{cfg.get('dataset')}.json".replace("/", "_")
        (out / name).write_text(json.dumps(r, indent=2))
    (out / "all_eval_results.json").write_text(json.dumps(cleaned, indent=2))
    try:
        import pandas as pd

        pd.json_normalize(cleaned).to_csv(out / "all_eval_results.csv", index=False)
    except ImportError:  # pandas is optional; the JSON files carry everything
        pass
    return {"individual_jsons": list(out.glob("*.json")), "combined_json": out / "all_eval_results.json",
            "csv": out / "all_eval_results.csv"}


def process_args(args: list[str]) -> argparse.Namespace:
    p = argparse.ArgumentParser(description="Run evaluations on SAEs")
    p.add_argument("sae_regex_pattern", type=str, help="regex over release names")
    p.add_argument("sae_block_pattern", type=str, help="regex over SAE ids")
    p.add_argument("--batch_size_prompts", type=int, default=16)
    p.add_argument("--n_eval_reconstruction_batches", type=int, default=10)
    p.add_argument("--compute_kl", action="store_true")
    p.add_argument("--compute_ce_loss", action="store_true")
    p.add_argument("--n_eval_sparsity_variance_batches", type=int, default=1)
    p.add_argument("--compute_l2_norms", action="store_true")
    p.add_argument("--compute_sparsity_metrics", action="store_true")
    p.add_argument("--compute_variance_metrics", action="store_true")
    p.add_argument("--compute_featurewise_density_statistics", action="store_true")
    p.add_argument("--compute_featurewise_weight_based_metrics", action="store_true")
    p.add_argument("--datasets", nargs="+", default=["Skylion007/openwebtext"])
    p.add_argument("--dataset_trust_remote_code", action="store_true")
    p.add_argument("--ctx_lens", nargs="+", type=int, default=[128])
    p.add_argument("--output_dir", type=str, default="eval_results")
    p.add_argument("--verbose", action="store_true")
    return p.parse_args(args)


def run_evals_cli(args: list[str] | None = None) -> None:
    import sys

    opts = process_args(sys.argv[1:] if args is None else args)
    files = process_results(run_evaluations(opts), opts.output_dir)
    print("Evaluation complete. Output files:")
    print(f"Individual JSONs: {len(files['individual_jsons'])}")
    print(f"Combined JSON: {files['combined_json']}")
    print(f"CSV: {files['csv']}")


if __name__ == "__main__":
    run_evals_cli()
