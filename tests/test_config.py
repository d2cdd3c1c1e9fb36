"""Runner configs: validation, defaults and dict round trips (behaviour of sae_lens/config.py;
cases follow tests/training/test_config.py)."""

import pytest

from saelens_b200.config import (
    CacheActivationsRunnerConfig,
    LanguageModelSAERunnerConfig,
    _default_cached_activations_path,
    json_dict,
    special_token,
)
from saelens_b200.models.jumprelu import JumpReLUTrainingSAEConfig
from saelens_b200.models.standard import StandardTrainingSAEConfig

SEQPOS_ERRORS = [(None, 10, -1), (None, 10, 0), (5, 5, None), (6, 3, None)]


@pytest.mark.parametrize("seqpos", SEQPOS_ERRORS)
def test_runner_config_rejects_bad_seqpos(seqpos):
    with pytest.raises(ValueError):
        LanguageModelSAERunnerConfig(sae=StandardTrainingSAEConfig(d_in=10, d_sae=10), seqpos_slice=seqpos,
                                     context_size=10)


@pytest.mark.parametrize("seqpos", SEQPOS_ERRORS)
def test_cache_config_rejects_bad_seqpos(seqpos):
    with pytest.raises(ValueError):
        CacheActivationsRunnerConfig(dataset_path="", model_name="", model_batch_size=1, hook_name="", d_in=1,
                                     training_tokens=100, context_size=10, seqpos_slice=seqpos)


def test_runner_config_accepts_valid_seqpos():
    cfg = LanguageModelSAERunnerConfig(sae=StandardTrainingSAEConfig(d_in=10, d_sae=10), seqpos_slice=(2, 8),
                                       context_size=10)
    assert cfg.seqpos_slice == (2, 8)


def test_hook_eval_is_deprecated():
    with pytest.warns(DeprecationWarning, match="The 'hook_eval' field is deprecated and will be removed in v7.0.0. "):
        LanguageModelSAERunnerConfig(sae=StandardTrainingSAEConfig(d_in=10, d_sae=10),
                                     hook_eval="blocks.0.hook_output")


def test_cache_config_context_larger_than_training_tokens():
    with pytest.raises(ValueError, match=r"context_size \(1024\) is greater than training_tokens \(100\)"):
        CacheActivationsRunnerConfig(dataset_path="", model_name="", model_batch_size=1, hook_name="", d_in=1,
                                     training_tokens=100, context_size=1024)


def test_default_cached_activations_path():
    assert _default_cached_activations_path("ds_path", "model_name", "hook_name", None) == \
        "activations/ds_path/model_name/hook_name"
    assert _default_cached_activations_path("ds_path", "model_name", "hook_name", 5) == \
        "activations/ds_path/model_name/hook_name_5"
    # slashes in hub names do not create directories
    assert _default_cached_activations_path("org/ds", "org/model", "h", None) == "activations/org_ds/org_model/h"


def test_use_cached_activations_fills_default_path():
    cfg = LanguageModelSAERunnerConfig(sae=StandardTrainingSAEConfig(d_in=10, d_sae=10), use_cached_activations=True,
                                       dataset_path="ds", model_name="m", hook_name="blocks.0.hook_resid_pre")
    assert cfg.cached_activations_path == "activations/ds/m/blocks.0.hook_resid_pre"


def test_runner_config_dict_roundtrip():
    cfg = LanguageModelSAERunnerConfig(
        sae=JumpReLUTrainingSAEConfig(d_in=5, d_sae=10, jumprelu_init_threshold=0.1, jumprelu_bandwidth=0.1,
                                      jumprelu_sparsity_loss_mode="tanh"),
        seqpos_slice=(0, 10), context_size=10)
    d = cfg.to_dict()
    assert d == cfg.to_dict()
    assert LanguageModelSAERunnerConfig.from_dict(d) == cfg


def test_from_dict_requires_fields():
    cfg = LanguageModelSAERunnerConfig(sae=StandardTrainingSAEConfig(d_in=5, d_sae=10), seqpos_slice=(0, 10),
                                       context_size=10)
    d = cfg.to_dict()
    del d["sae"]
    with pytest.raises(ValueError, match="sae field is required in the config dictionary"):
        LanguageModelSAERunnerConfig.from_dict(d)
    d = cfg.to_dict()
    del d["sae"]["architecture"]
    with pytest.raises(ValueError, match="architecture field is required in the sae dictionary"):
        LanguageModelSAERunnerConfig.from_dict(d)
    d = cfg.to_dict()
    del d["logger"]
    with pytest.raises(ValueError, match="logger field is required in the config dictionary"):
        LanguageModelSAERunnerConfig.from_dict(d)


def test_json_dict():
    assert json_dict('{"key": "value"}') == {"key": "value"}
    assert json_dict("{}") == {}
    assert json_dict("null") is None
    for bad in ("[1, 2, 3]", '"just a string"', "123"):
        with pytest.raises(ValueError, match="Expected a dictionary"):
            json_dict(bad)


def test_special_token():
    for s in ("none", "None", "NONE"):
        assert special_token(s) is None
    for s in ("bos", "eos", "sep"):
        assert special_token(s) == s
    assert special_token("0") == 0 and special_token("42") == 42 and special_token("-1") == -1
    for bad in ("invalid", "foo"):
        with pytest.raises(ValueError, match="Expected 'bos', 'eos', 'sep', an integer"):
            special_token(bad)


def test_exclude_special_tokens_must_be_ints():
    with pytest.raises(ValueError, match="exclude_special_tokens list must contain only integers"):
        LanguageModelSAERunnerConfig(sae=StandardTrainingSAEConfig(d_in=10, d_sae=10),
                                     exclude_special_tokens=["not", "integers"])


def test_derived_fields():
    cfg = LanguageModelSAERunnerConfig(sae=StandardTrainingSAEConfig(d_in=10, d_sae=20), lr=1e-3,
                                       train_batch_size_tokens=64, context_size=8, n_batches_in_buffer=4,
                                       training_tokens=6400)
    assert cfg.lr_end == pytest.approx(1e-4)
    assert cfg.tokens_per_buffer == 64 * 8 * 4
    assert cfg.total_training_steps == 100
    assert cfg.logger.run_name.startswith("standard-20-LR-0.001")


def test_runner_config_rejects_negative_context():
    with pytest.raises(ValueError, match="negative"):
        LanguageModelSAERunnerConfig(sae=StandardTrainingSAEConfig(d_in=10, d_sae=10), context_size=-1)


def test_history_intervals_need_output_path():
    with pytest.raises(ValueError, match="requires output_path"):
        LanguageModelSAERunnerConfig(sae=StandardTrainingSAEConfig(d_in=10, d_sae=10), save_mse_every_n_steps=5,
                                     output_path=None)
    with pytest.raises(ValueError, match=">= 0"):
        LanguageModelSAERunnerConfig(sae=StandardTrainingSAEConfig(d_in=10, d_sae=10), save_timing_every_n_steps=-1,
                                     output_path="x")


def test_compile_sae_incompatible_with_ddp():
    with pytest.raises(ValueError, match="compile_sae=True is incompatible"):
        LanguageModelSAERunnerConfig(sae=StandardTrainingSAEConfig(d_in=10, d_sae=10), sae_dp_mode="ddp",
                                     compile_sae=True)
