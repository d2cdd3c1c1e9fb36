"""End-to-end CPU runs: LM -> activations store -> trainer -> saved SAE, CLI parsing, evals,
HookedSAETransformer splicing, sequence packing."""

import json

import pytest
import torch

from saelens_b200 import SAE, SAEMetadata, StandardSAE, StandardSAEConfig, StandardTrainingSAEConfig, TopKTrainingSAEConfig
from saelens_b200.config import LanguageModelSAERunnerConfig, LoggingConfig
from saelens_b200.models.lm import HookedLM, preset_config
from saelens_b200.training.activations_store import ActivationsStore
from saelens_b200.training.tokenization_and_batching import concat_and_batch_sequences


def _tiny_lm():
    torch.manual_seed(0)
    return HookedLM(preset_config("gpt2", n_layers=2, d_model=64, n_heads=4, d_mlp=128, d_vocab=500, n_ctx=64,
                                  dtype="float32"))


def _cfg(tmp_path, arch="standard", **kw):
    sae = (StandardTrainingSAEConfig(d_in=64, d_sae=128, l1_coefficient=1e-3) if arch == "standard"
           else TopKTrainingSAEConfig(d_in=64, d_sae=128, k=8))
    base = dict(sae=sae, model_name="gpt2", hook_name="blocks.1.hook_resid_pre", dataset_path="synthetic:uniform:500:32",
                context_size=16, training_tokens=64 * 30, train_batch_size_tokens=64, store_batch_size_prompts=4,
                n_batches_in_buffer=2, checkpoint_path=str(tmp_path / "ckpt"), output_path=str(tmp_path / "out"),
                logger=LoggingConfig(log_to_wandb=False), device="cpu", save_mse_every_n_steps=1, n_checkpoints=1,
                verbose=False)
    base.update(kw)
    return LanguageModelSAERunnerConfig(**base)


def test_packing_rules():
    seqs = [torch.tensor([5, 6, 7]), torch.tensor([8, 9]), torch.tensor([10, 11, 12, 13])]
    out = [t.tolist() for t in concat_and_batch_sequences(iter(seqs), 4, begin_batch_token_id=1,
                                                          sequence_separator_token_id=2)]
    assert out == [[1, 5, 6, 7], [1, 8, 9, 2], [1, 10, 11, 12]]
    out = [t.tolist() for t in concat_and_batch_sequences(iter(seqs), 3, begin_batch_token_id=1,
                                                          disable_concat_sequences=True)]
    assert out == [[1, 5, 6], [1, 8, 9], [1, 10, 11]]


def test_activations_store_shapes_and_resume(tmp_path):
    lm = _tiny_lm()
    store = ActivationsStore.from_config(lm, _cfg(tmp_path))
    toks = store.get_batch_tokens()
    assert toks.shape == (4, 16)
    acts = store.get_activations(toks)
    assert acts.shape == (4, 16, 64)
    _, cache = lm.run_with_cache(toks, names_filter="blocks.1.hook_resid_pre")
    assert torch.allclose(acts, cache["blocks.1.hook_resid_pre"])
    b = next(store)
    assert b.shape == (64, 64)
    store.save_to_checkpoint(tmp_path)
    s2 = ActivationsStore.from_config(lm, _cfg(tmp_path))
    s2.load_from_checkpoint(tmp_path)
    assert s2.n_dataset_processed == store.n_dataset_processed > 0


@pytest.mark.parametrize("arch", ["standard", "topk"])
def test_runner_end_to_end_cpu(tmp_path, arch):
    from saelens_b200.runners.llm_sae_training_runner import LanguageModelSAETrainingRunner

    cfg = _cfg(tmp_path, arch=arch)
    runner = LanguageModelSAETrainingRunner(cfg, override_model=_tiny_lm())
    sae = runner.run()
    out = tmp_path / "out"
    assert (out / "cfg.json").exists() and (out / "sae_weights.safetensors").exists()
    assert (out / "runner_cfg.json").exists() and (out / "sparsity.safetensors").exists()
    loaded = SAE.load_from_disk(out)
    assert loaded.cfg.d_sae == 128 and loaded.cfg.metadata.hook_name == "blocks.1.hook_resid_pre"
    rows = [json.loads(x) for x in (out / "mse_history.jsonl").read_text().splitlines()]
    assert len(rows) == 30 and rows[-1]["mse_loss"] < rows[0]["mse_loss"]
    ck = list((tmp_path / "ckpt").rglob("trainer_state.pt"))
    assert ck, "expected one intermediate checkpoint"
    assert (ck[0].parent / "activations_store_state.safetensors").exists()
    del sae


def test_cli_parsing():
    from saelens_b200.runners.llm_sae_training_runner import _parse_cfg_args

    cfg = _parse_cfg_args(["--architecture", "topk", "--d_in", "64", "--d_sae", "256", "--k", "16",
                           "--model_name", "gpt2", "--hook_name", "blocks.0.hook_resid_pre", "--lr", "1e-3",
                           "--log_to_wandb", "false", "--checkpoint_path", "none", "--verbose", "false"])
    assert cfg.sae.architecture() == "topk" and cfg.sae.k == 16 and cfg.lr == 1e-3
    assert cfg.logger.log_to_wandb is False and cfg.checkpoint_path is None


def test_run_evals_metrics(tmp_path):
    from saelens_b200.evals import get_eval_everything_config, run_evals

    lm = _tiny_lm()
    store = ActivationsStore.from_config(lm, _cfg(tmp_path))
    sae = StandardSAE(StandardSAEConfig(d_in=64, d_sae=128, metadata=SAEMetadata(hook_name="blocks.1.hook_resid_pre")))
    metrics, feat = run_evals(sae, store, lm, get_eval_everything_config(4, 1, 1))
    assert {"model_behavior_preservation", "model_performance_preservation", "reconstruction_quality",
            "shrinkage", "sparsity", "token_stats"} <= set(metrics)
    assert len(feat["feature_density"]) == 128
    # an SAE with identity-like reconstruction has ce_loss_score ~ 1
    id_sae = StandardSAE(StandardSAEConfig(d_in=64, d_sae=128, metadata=SAEMetadata(hook_name="blocks.1.hook_resid_pre")))
    with torch.no_grad():
        id_sae.W_enc.zero_(); id_sae.W_dec.zero_()
        id_sae.W_enc[:, :64] = torch.eye(64); id_sae.W_enc[:, 64:] = -torch.eye(64)
        id_sae.W_dec[:64] = torch.eye(64); id_sae.W_dec[64:] = -torch.eye(64)
    m2, _ = run_evals(id_sae, store, lm, get_eval_everything_config(4, 1, 1))
    assert m2["model_performance_preservation"]["ce_loss_score"] == pytest.approx(1.0, abs=1e-4)
    assert m2["reconstruction_quality"]["explained_variance"] == pytest.approx(1.0, abs=1e-5)


def test_runner_multi_hook_trains_one_sae_per_hook(tmp_path):
    from saelens_b200.runners.llm_sae_training_runner import LanguageModelSAETrainingRunner
    from saelens_b200.training.multi_sae_trainer import sanitize_hook_name_for_path

    hooks = ["blocks.0.hook_resid_pre", "blocks.1.hook_resid_pre"]
    cfg = _cfg(tmp_path, hook_names=hooks, training_tokens=64 * 10, multi_sae_seed_mode="offset")
    runner = LanguageModelSAETrainingRunner(cfg, override_model=_tiny_lm())
    out_saes = runner.run()
    assert set(out_saes) == set(hooks)
    w = [out_saes[h].W_dec.detach().clone() for h in hooks]
    assert not torch.equal(w[0], w[1])  # offset seeds and different inputs
    for h in hooks:
        d = tmp_path / "out" / sanitize_hook_name_for_path(h)
        loaded = SAE.load_from_disk(d)
        assert loaded.cfg.metadata.hook_name == h and loaded.cfg.d_sae == 128
    assert runner.trainer.n_training_steps == 10
    assert (tmp_path / "out" / "runner_cfg.json").exists()


def test_runner_compile_flags(tmp_path, monkeypatch):
    from saelens_b200.runners.llm_sae_training_runner import LanguageModelSAETrainingRunner

    calls = []

    def fake_compile(fn, mode=None, **kw):
        calls.append((getattr(fn, "__name__", type(fn).__name__), mode))
        return fn

    monkeypatch.setattr(torch, "compile", fake_compile)
    cfg = _cfg(tmp_path, compile_llm=True, llm_compilation_mode="max-autotune-no-cudagraphs", compile_sae=True,
               sae_compilation_mode="max-autotune")
    LanguageModelSAETrainingRunner(cfg, override_model=_tiny_lm())
    assert ("HookedLM", "max-autotune-no-cudagraphs") in calls
    assert ("training_forward_pass", "max-autotune") in calls
