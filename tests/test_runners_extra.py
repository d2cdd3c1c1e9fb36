"""CacheActivationsRunner -> cached-activation training, PretokenizeRunner, MultiSAETrainer."""

import json

import numpy as np
import pytest
import torch

from saelens_b200.config import CacheActivationsRunnerConfig, LoggingConfig, PretokenizeRunnerConfig, SAETrainerConfig
from saelens_b200.models.lm import HookedLM, preset_config
from saelens_b200.models.standard import StandardTrainingSAE, StandardTrainingSAEConfig
from saelens_b200.models.topk import TopKTrainingSAE, TopKTrainingSAEConfig
from saelens_b200.runners.cache_activations_runner import CacheActivationsRunner
from saelens_b200.runners.pretokenize_runner import PretokenizeRunner
from saelens_b200.training.activations_store import ActivationsStore
from saelens_b200.training.multi_sae_trainer import MultiSAETrainer


def _lm():
    torch.manual_seed(0)
    return HookedLM(preset_config("gpt2", n_layers=2, d_model=64, n_heads=4, d_mlp=128, d_vocab=500, n_ctx=64,
                                  dtype="float32"))


def test_cache_activations_roundtrip(tmp_path):
    cfg = CacheActivationsRunnerConfig(dataset_path="synthetic:uniform:500:32", model_name="gpt2", model_batch_size=4,
                                       hook_name="blocks.0.hook_resid_post", d_in=64, training_tokens=16 * 40,
                                       context_size=16, new_cached_activations_path=str(tmp_path / "cache"),
                                       device="cpu", buffer_size_gb=16 * 10 * 64 * 4 / 1e9, shuffle=False)
    lm = _lm()
    out = CacheActivationsRunner(cfg, override_model=lm).run()
    info = json.loads((out / "cache_info.json").read_text())
    assert info["total_tokens"] == 16 * 40 and info["n_shards"] == len(list(out.glob("*.safetensors"))) > 1
    from safetensors.torch import load_file

    sd = load_file(str(sorted(out.glob("*.safetensors"))[0]))
    toks = sd["token_ids"][:2].long()
    _, cache = lm.run_with_cache(toks, names_filter="blocks.0.hook_resid_post")
    assert torch.allclose(sd["activations"][:2], cache["blocks.0.hook_resid_post"], atol=1e-5)
    store = ActivationsStore(model=lm, dataset=None, hook_name="blocks.0.hook_resid_post", context_size=16, d_in=64,
                             n_batches_in_buffer=2, total_training_tokens=640, store_batch_size_prompts=4,
                             train_batch_size_tokens=32, cached_activations_path=str(out), activations_mixing_fraction=0)
    assert next(store).shape == (32, 64)


class _Tok:
    bos_token_id, eos_token_id, sep_token_id = 1, 2, 3

    def encode(self, s):
        return [10 + (ord(c) % 50) for c in s]


def test_pretokenize(tmp_path):
    cfg = PretokenizeRunnerConfig(tokenizer_name="char", context_size=8, save_path=str(tmp_path / "pt"), shuffle=False)
    data = [{"text": "hello world"}, {"text": "sparse autoencoders"}, {"text": "b200"}]
    out = PretokenizeRunner(cfg, tokenizer=_Tok(), override_dataset=data).run()
    arr = np.load(out / "tokens.npy")
    assert arr.shape[1] == 8 and (arr[:, 0] == 1).all()
    meta = json.loads((out / "sae_lens.json").read_text())
    assert meta["context_size"] == 8 and meta["n_rows"] == len(arr)


def test_multi_sae_trainer_two_hooks(tmp_path):
    cfg = SAETrainerConfig(
        n_checkpoints=0, checkpoint_path=None, save_final_checkpoint=False, output_path=None, save_mse_every_n_steps=0,
        save_timing_every_n_steps=0, save_memory_every_n_steps=0, synchronize_timing=False,
        multi_sae_backward_order="largest_first", multi_sae_stats_sync_mode="immediate", multi_sae_stats_sync_interval=1,
        total_training_samples=32 * 20, device="cpu", autocast=False, lr=1e-3, lr_end=1e-4,
        lr_scheduler_name="constant", lr_warm_up_steps=0, adam_beta1=0.9, adam_beta2=0.999, lr_decay_steps=0,
        n_restart_cycles=1, train_batch_size_samples=32, dead_feature_window=5, feature_sampling_window=10,
        logger=LoggingConfig(log_to_wandb=False))
    saes = {"a": StandardTrainingSAE(StandardTrainingSAEConfig(d_in=16, d_sae=32)),
            "b": TopKTrainingSAE(TopKTrainingSAEConfig(d_in=16, d_sae=64, k=4))}
    g = torch.Generator().manual_seed(0)

    def gen():
        while True:
            yield {"a": torch.randn(32, 16, generator=g), "b": torch.randn(32, 16, generator=g)}

    for mode in ("combined", "sequential"):
        tr = MultiSAETrainer(hook_names=["a", "b"], sae_by_hook=saes, data_provider=gen(), cfg=cfg, backward_mode=mode)
        tr.fit()
        assert tr.n_training_steps == 20
    tr.save_final(tmp_path / "final")
    tr.save_checkpoint(tmp_path / "ck")
    man = json.loads((tmp_path / "final" / "multi_sae_manifest.json").read_text())
    assert man["hook_names"] == ["a", "b"]
    tr2 = MultiSAETrainer(hook_names=["a", "b"], sae_by_hook=saes, data_provider=gen(), cfg=cfg)
    tr2.load_trainer_state(tmp_path / "ck")
    assert tr2.n_training_steps == 20


def test_pretokenize_shuffle_and_streaming_checks(tmp_path):
    data = [{"text": "hello world " * 3}, {"text": "sparse autoencoders " * 3}, {"text": "b200 " * 6}]
    plain = PretokenizeRunner(PretokenizeRunnerConfig(tokenizer_name="char", context_size=8, shuffle=False),
                              tokenizer=_Tok(), override_dataset=data).tokenize()
    mixed = PretokenizeRunner(PretokenizeRunnerConfig(tokenizer_name="char", context_size=8, shuffle=True, seed=3),
                              tokenizer=_Tok(), override_dataset=data).tokenize()
    # shuffling permutes whole contexts
    assert sorted(map(tuple, plain.tolist())) == sorted(map(tuple, mixed.tolist()))
    cfg = PretokenizeRunnerConfig(tokenizer_name="char", context_size=8, num_proc=2, streaming=True)
    with pytest.raises(ValueError, match="num_proc must be 1"):
        PretokenizeRunner(cfg, tokenizer=_Tok(), override_dataset=data).tokenize()


def _cache_cfg(tmp_path, **kw):
    base = dict(dataset_path="synthetic:uniform:500:32", model_name="gpt2", model_batch_size=4,
                hook_name="blocks.0.hook_resid_post", d_in=64, training_tokens=16 * 8, context_size=16,
                new_cached_activations_path=str(tmp_path / "cache"), device="cpu",
                buffer_size_gb=16 * 8 * 64 * 4 / 1e9, shuffle=False)
    base.update(kw)
    return CacheActivationsRunnerConfig(**base)


def test_cache_runner_refuses_a_nonempty_directory_and_a_wrong_width(tmp_path):
    (tmp_path / "cache").mkdir()
    (tmp_path / "cache" / "some_file.txt").write_text("keep me")
    with pytest.raises(FileExistsError, match="is not empty. Please delete it or specify a different path."):
        CacheActivationsRunner(_cache_cfg(tmp_path), override_model=_lm()).run()
    assert (tmp_path / "cache" / "some_file.txt").read_text() == "keep me"
    with pytest.raises(RuntimeError, match="has width 64, but d_in is 65"):
        CacheActivationsRunner(_cache_cfg(tmp_path, d_in=65, new_cached_activations_path=str(tmp_path / "c2")),
                               override_model=_lm()).run()


def test_cache_runner_seqpos_and_shuffle_keep_token_alignment(tmp_path):
    lm = _lm()
    out = CacheActivationsRunner(_cache_cfg(tmp_path, seqpos_slice=(2, 10), shuffle=True), override_model=lm).run()
    from safetensors.torch import load_file

    sd = load_file(str(sorted(out.glob("*.safetensors"))[0]))
    assert sd["activations"].shape[1] == 8 and sd["token_ids"].shape[1] == 8
    # shuffled positions still carry their own token id: same multiset as an unshuffled run
    plain = CacheActivationsRunner(_cache_cfg(tmp_path, seqpos_slice=(2, 10), shuffle=False,
                                              new_cached_activations_path=str(tmp_path / "plain")),
                                   override_model=lm).run()
    sp = load_file(str(sorted(plain.glob("*.safetensors"))[0]))
    assert sorted(sd["token_ids"].flatten().tolist()) == sorted(sp["token_ids"].flatten().tolist())


def test_multi_sae_checkpoint_restores_state_and_rejects_other_hooks(tmp_path):
    cfg = SAETrainerConfig(
        n_checkpoints=0, checkpoint_path=None, save_final_checkpoint=False, output_path=None, save_mse_every_n_steps=0,
        save_timing_every_n_steps=0, save_memory_every_n_steps=0, synchronize_timing=False,
        multi_sae_backward_order="forward", multi_sae_stats_sync_mode="immediate", multi_sae_stats_sync_interval=1,
        total_training_samples=32 * 6, device="cpu", autocast=False, lr=1e-3, lr_end=1e-4,
        lr_scheduler_name="constant", lr_warm_up_steps=0, adam_beta1=0.9, adam_beta2=0.999, lr_decay_steps=0,
        n_restart_cycles=1, train_batch_size_samples=32, dead_feature_window=5, feature_sampling_window=10,
        logger=LoggingConfig(log_to_wandb=False))
    g = torch.Generator().manual_seed(0)

    def gen():
        while True:
            yield {"a": torch.randn(32, 16, generator=g), "b": torch.randn(32, 16, generator=g)}

    saes = {"a": StandardTrainingSAE(StandardTrainingSAEConfig(d_in=16, d_sae=32)),
            "b": StandardTrainingSAE(StandardTrainingSAEConfig(d_in=16, d_sae=32))}
    tr = MultiSAETrainer(hook_names=["a", "b"], sae_by_hook=saes, data_provider=gen(), cfg=cfg)
    tr.fit()
    tr.save_checkpoint(tmp_path / "ck")
    tr2 = MultiSAETrainer(hook_names=["a", "b"], sae_by_hook=saes, data_provider=gen(), cfg=cfg)
    tr2.load_trainer_state(tmp_path / "ck")
    assert tr2.n_training_samples == tr.n_training_samples
    for h in ("a", "b"):
        torch.testing.assert_close(tr2.act_freq_scores[h], tr.act_freq_scores[h])
    s1, s2 = tr.optimizer.state_dict()["state"], tr2.optimizer.state_dict()["state"]
    assert s1.keys() == s2.keys() and all(torch.equal(s1[k]["exp_avg"], s2[k]["exp_avg"]) for k in s1)
    other = {"a": saes["a"], "c": StandardTrainingSAE(StandardTrainingSAEConfig(d_in=16, d_sae=32))}
    tr3 = MultiSAETrainer(hook_names=["a", "c"], sae_by_hook=other, data_provider=gen(), cfg=cfg)
    with pytest.raises(ValueError, match="do not match"):
        tr3.load_trainer_state(tmp_path / "ck")
