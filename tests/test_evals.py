"""SAE evaluation metrics and CLI helpers (behaviour of sae_lens/evals.py; cases follow
tests/test_evals.py)."""

import json
from unittest import mock

import pytest
import torch

from saelens_b200.config import LanguageModelSAERunnerConfig, LoggingConfig
from saelens_b200.evals import (
    EvalConfig,
    _kl,
    all_loadable_saes,
    get_eval_everything_config,
    get_saes_from_regex,
    get_sparsity_and_variance_metrics,
    process_args,
    process_results,
    run_evals,
)
from saelens_b200.models.lm.transformer import HookedLM, preset_config
from saelens_b200.models.sae import SAEMetadata
from saelens_b200.models.standard import StandardSAE, StandardSAEConfig
from saelens_b200.models.topk import TopKSAE, TopKSAEConfig
from saelens_b200.training.activation_scaler import ActivationScaler
from saelens_b200.training.activations_store import ActivationsStore
from saelens_b200.models.standard import StandardTrainingSAEConfig

HOOK = "blocks.1.hook_resid_pre"


@pytest.fixture(scope="module")
def lm():
    torch.manual_seed(0)
    return HookedLM(preset_config("gpt2", n_layers=2, d_model=32, n_heads=4, d_mlp=64, d_vocab=200, n_ctx=32,
                                  dtype="float32"))


def _store(lm, tmp_path):
    cfg = LanguageModelSAERunnerConfig(
        sae=StandardTrainingSAEConfig(d_in=32, d_sae=64), model_name="gpt2", hook_name=HOOK,
        dataset_path="synthetic:uniform:200:16", context_size=16, training_tokens=64 * 10, train_batch_size_tokens=64,
        store_batch_size_prompts=4, n_batches_in_buffer=2, checkpoint_path=None, output_path=None,
        logger=LoggingConfig(log_to_wandb=False), device="cpu", verbose=False)
    return ActivationsStore.from_config(lm, cfg)


def _sae(kind="standard"):
    torch.manual_seed(1)
    md = SAEMetadata(hook_name=HOOK)
    sae = (TopKSAE(TopKSAEConfig(d_in=32, d_sae=64, k=4, metadata=md)) if kind == "topk"
           else StandardSAE(StandardSAEConfig(d_in=32, d_sae=64, metadata=md)))
    with torch.no_grad():
        for p in sae.parameters():
            p.copy_(torch.randn_like(p) * 0.2)
    return sae


def _identity_sae():
    sae = StandardSAE(StandardSAEConfig(d_in=32, d_sae=64, metadata=SAEMetadata(hook_name=HOOK)))
    with torch.no_grad():
        for p in sae.parameters():
            p.zero_()
        sae.W_enc[:, :32] = torch.eye(32)
        sae.W_enc[:, 32:] = -torch.eye(32)
        sae.W_dec[:32] = torch.eye(32)
        sae.W_dec[32:] = -torch.eye(32)
    return sae


GROUPS = {"model_behavior_preservation", "model_performance_preservation", "reconstruction_quality", "shrinkage",
          "sparsity", "token_stats"}


@pytest.mark.parametrize("kind", ["standard", "topk"])
def test_run_evals_reports_every_group(lm, tmp_path, kind):
    store = _store(lm, tmp_path)
    metrics, feat = run_evals(_sae(kind), store, lm, ActivationScaler(), get_eval_everything_config(4, 2, 2))
    assert set(metrics) == GROUPS
    assert set(metrics["model_behavior_preservation"]) == {"kl_div_score", "kl_div_with_ablation", "kl_div_with_sae"}
    assert set(metrics["model_performance_preservation"]) == {"ce_loss_score", "ce_loss_with_ablation",
                                                              "ce_loss_with_sae", "ce_loss_without_sae"}
    assert set(metrics["reconstruction_quality"]) == {"explained_variance", "explained_variance_legacy", "mse",
                                                      "cossim"}
    assert set(metrics["shrinkage"]) == {"l2_norm_in", "l2_norm_out", "l2_ratio", "relative_reconstruction_bias"}
    assert set(metrics["sparsity"]) == {"l0", "l1"}
    assert metrics["token_stats"] == {"total_tokens_eval_reconstruction": 16 * 2 * 4,
                                      "total_tokens_eval_sparsity_variance": 16 * 2 * 4}
    assert {"feature_density", "consistent_activation_heuristic", "encoder_norm", "encoder_decoder_cosine_sim",
            "encoder_bias"} == set(feat)
    assert all(len(v) == 64 for v in feat.values())
    if kind == "topk":
        assert metrics["sparsity"]["l0"] <= 4 + 1e-6


def test_identity_sae_is_a_perfect_reconstruction(lm, tmp_path):
    metrics, _ = run_evals(_identity_sae(), _store(lm, tmp_path), lm, ActivationScaler(),
                           get_eval_everything_config(4, 1, 2))
    assert metrics["reconstruction_quality"]["explained_variance"] == pytest.approx(1.0, abs=1e-5)
    assert metrics["reconstruction_quality"]["mse"] == pytest.approx(0.0, abs=1e-8)
    assert metrics["reconstruction_quality"]["cossim"] == pytest.approx(1.0, abs=1e-5)
    assert metrics["shrinkage"]["l2_ratio"] == pytest.approx(1.0, abs=1e-5)
    assert metrics["shrinkage"]["relative_reconstruction_bias"] == pytest.approx(1.0, abs=1e-5)
    assert metrics["model_performance_preservation"]["ce_loss_score"] == pytest.approx(1.0, abs=1e-4)
    assert metrics["model_behavior_preservation"]["kl_div_with_sae"] == pytest.approx(0.0, abs=1e-6)


def test_empty_eval_config_gives_token_stats_only(lm, tmp_path):
    metrics, feat = run_evals(_sae(), _store(lm, tmp_path), lm, ActivationScaler(), EvalConfig())
    assert set(metrics) == {"token_stats"} and feat == {}


def test_zero_batches_rejected(lm, tmp_path):
    with pytest.raises(ValueError, match="n_eval_reconstruction_batches must be > 0"):
        run_evals(_sae(), _store(lm, tmp_path), lm, ActivationScaler(),
                  EvalConfig(compute_kl=True, n_eval_reconstruction_batches=0))
    with pytest.raises(ValueError, match="n_eval_sparsity_variance_batches must be > 0"):
        run_evals(_sae(), _store(lm, tmp_path), lm, ActivationScaler(),
                  EvalConfig(compute_l2_norms=True, n_eval_sparsity_variance_batches=0))


def test_ignored_tokens_are_excluded_and_left_clean(lm, tmp_path):
    store = _store(lm, tmp_path)
    toks = store.get_batch_tokens(4)
    store.reset_input_dataset()
    ignore = sorted(set(toks[:, :4].flatten().tolist()))
    cfg = get_eval_everything_config(4, 1, 1)
    m_all, f_all = run_evals(_sae(), store, lm, ActivationScaler(), cfg, exclude_special_tokens=False)
    store.reset_input_dataset()
    m_ign, f_ign = run_evals(_sae(), store, lm, ActivationScaler(), cfg, exclude_special_tokens=ignore)
    assert m_ign["sparsity"]["l0"] != pytest.approx(m_all["sparsity"]["l0"])
    # density is over the kept tokens only
    keep = ~torch.isin(toks, torch.tensor(ignore))
    sae = _sae()
    _, cache = lm.run_with_cache(toks, names_filter=[HOOK])
    f = sae.encode(cache[HOOK])
    want = ((f > 0) & keep.unsqueeze(-1)).float().sum((0, 1)) / keep.sum()
    torch.testing.assert_close(torch.tensor(f_ign["feature_density"]), want, atol=1e-6, rtol=1e-5)


def test_activation_scaler_is_applied_around_the_sae(lm, tmp_path):
    store = _store(lm, tmp_path)
    sae = _sae()
    cfg = EvalConfig(compute_sparsity_metrics=True, n_eval_sparsity_variance_batches=1, batch_size_prompts=4)
    m1, _ = get_sparsity_and_variance_metrics(sae, lm, store, ActivationScaler(2.0), 1, False, True, False, False, 4)
    store.reset_input_dataset()
    toks = store.get_batch_tokens(4)
    _, cache = lm.run_with_cache(toks, names_filter=[HOOK])
    want = (sae.encode(cache[HOOK] * 2.0) > 0).float().sum(-1).mean().item()
    assert m1["l0"] == pytest.approx(want)
    del cfg


def test_kl_formula():
    torch.manual_seed(0)
    a, b = torch.randn(2, 3, 7), torch.randn(2, 3, 7)
    p = torch.softmax(a, -1)
    want = (p * (torch.log(p) - torch.log_softmax(b, -1))).sum(-1)
    torch.testing.assert_close(_kl(a, b), want)
    torch.testing.assert_close(_kl(a, a), torch.zeros(2, 3), atol=1e-6, rtol=0)


def test_process_results_writes_json_and_csv(tmp_path):
    res = [{"unique_id": "rel-a/b", "eval_cfg": {"context_size": 8, "dataset": "org/ds"},
            "metrics": {"x": float("nan"), "y": 1.0}}]
    out = process_results(res, str(tmp_path))
    combined = json.loads(out["combined_json"].read_text())
    assert combined[0]["metrics"]["x"] == -1
    assert (tmp_path / "rel-a_b_8_org_ds.json").exists()
    assert out["csv"].exists()


def test_loadable_saes_and_regex():
    info = type("L", (), {"saes_map": {"blocks.0.hook_resid_pre": "p0", "blocks.1.hook_resid_pre": "p1"},
                          "expected_var_explained": {"blocks.0.hook_resid_pre": 0.9, "blocks.1.hook_resid_pre": 0.8},
                          "expected_l0": {"blocks.0.hook_resid_pre": 10.0, "blocks.1.hook_resid_pre": 20.0}})()
    with mock.patch("saelens_b200.loading.pretrained_saes_directory.get_pretrained_saes_directory",
                    return_value={"rel-a": info, "other": info}):
        allx = all_loadable_saes()
        assert ("rel-a", "blocks.0.hook_resid_pre", 0.9, 10.0) in allx and len(allx) == 4
        assert get_saes_from_regex("rel-a", r"blocks\.1\..*") == [("rel-a", "blocks.1.hook_resid_pre", 0.8, 20.0)]
        assert get_saes_from_regex("nothing", ".*") == []
        assert len(get_saes_from_regex(".*", ".*")) == 4


def test_process_args_defaults_and_flags():
    a = process_args(["gpt2-small-res-jb", "blocks.0.hook_resid_pre", "--compute_kl", "--ctx_lens", "64", "128"])
    assert a.sae_regex_pattern == "gpt2-small-res-jb" and a.compute_kl and not a.compute_ce_loss
    assert a.ctx_lens == [64, 128] and a.batch_size_prompts == 16 and a.datasets == ["Skylion007/openwebtext"]
    assert a.output_dir == "eval_results"


def test_training_evaluator_keeps_the_training_token_position(lm, tmp_path):
    from saelens_b200.evals import LLMSaeEvaluator

    store = _store(lm, tmp_path)
    store.get_batch_tokens(4)
    before = store.n_dataset_processed
    nxt = store.get_batch_tokens(4)
    store2 = _store(lm, tmp_path)
    store2.get_batch_tokens(4)
    out = LLMSaeEvaluator(lm, store2, 1, 4)(_sae(), None, ActivationScaler())
    assert "eval/sparsity/l0" in out and store2.n_dataset_processed == before
    assert torch.equal(store2.get_batch_tokens(4), nxt)
