"""ActivationsStore (behaviour of sae_lens/training/activations_store.py; cases follow
tests/training/test_activations_store.py): shapes, head hooks, position slices, special-token
filtering, pretokenized length checks, strided sharding, checkpoints."""

import pytest
import torch

from saelens_b200.models.lm.transformer import HookedLM, preset_config
from saelens_b200.models.sae import SAEMetadata
from saelens_b200.models.standard import StandardSAE, StandardSAEConfig
from saelens_b200.training.activations_store import ActivationsStore

HOOK = "blocks.1.hook_resid_pre"


@pytest.fixture(scope="module")
def lm():
    torch.manual_seed(0)
    return HookedLM(preset_config("gpt2", n_layers=2, d_model=32, n_heads=4, d_mlp=64, d_vocab=200, n_ctx=32,
                                  dtype="float32"))


def _store(lm, dataset="synthetic:uniform:200:16", **kw):
    args = dict(model=lm, dataset=dataset, hook_name=HOOK, context_size=16, d_in=32, n_batches_in_buffer=2,
                total_training_tokens=10**6, store_batch_size_prompts=4, train_batch_size_tokens=32, prepend_bos=False)
    args.update(kw)
    return ActivationsStore(**args)


def test_shapes_and_activations_match_the_model(lm):
    s = _store(lm)
    toks = s.get_batch_tokens()
    assert toks.shape == (4, 16)
    acts = s.get_activations(toks)
    _, cache = lm.run_with_cache(toks, names_filter=HOOK)
    torch.testing.assert_close(acts, cache[HOOK])
    b = next(s)
    assert b.shape == (32, 32)


def test_head_hook_selects_one_head(lm):
    s = _store(lm, hook_name="blocks.0.attn.hook_z", hook_head_index=2, d_in=8)
    toks = s.get_batch_tokens()
    _, cache = lm.run_with_cache(toks, names_filter="blocks.0.attn.hook_z")
    torch.testing.assert_close(s.get_activations(toks), cache["blocks.0.attn.hook_z"][:, :, 2])


def test_position_slice_keeps_only_those_positions(lm):
    s = _store(lm, seqpos_slice=(2, 10))
    toks = s.get_batch_tokens()
    acts = s.get_activations(toks)
    assert acts.shape == (4, 8, 32)
    _, cache = lm.run_with_cache(toks, names_filter=HOOK)
    torch.testing.assert_close(acts, cache[HOOK][:, 2:10])


def test_special_tokens_are_filtered_from_batches(lm):
    rows = torch.randint(5, 200, (40, 16))
    rows[:, 0] = 1  # a "special" token at every context start
    s = _store(lm, dataset=rows, exclude_special_tokens=[1])
    b = s.get_filtered_llm_batch()
    assert b.shape[0] == 4 * 15  # one position per context dropped
    s2 = _store(lm, dataset=rows)
    assert s2.get_filtered_llm_batch().shape[0] == 4 * 16


@pytest.mark.parametrize("ctx,expect", [(8, "warn"), (10, None), (12, "error")])
def test_pretokenized_length_against_context_size(lm, ctx, expect):
    rows = torch.randint(0, 200, (20, 10))
    if expect == "error":
        with pytest.raises(ValueError, match="pretokenized dataset has context size 10"):
            _store(lm, dataset=rows, context_size=ctx)
    elif expect == "warn":
        with pytest.warns(RuntimeWarning):
            _store(lm, dataset=rows, context_size=ctx)
    else:
        _store(lm, dataset=rows, context_size=ctx)


def test_strided_sharding_splits_rows_without_overlap(lm):
    rows = torch.arange(48 * 16).reshape(48, 16)
    seen = []
    for shard in range(3):
        s = _store(lm, dataset=rows, shard_index=shard, num_shards=3)
        got = s.get_batch_tokens(16)
        seen.append({int(r[0]) // 16 for r in got})
        assert all(int(r[0]) // 16 % 3 == shard for r in got)
    assert not (seen[0] & seen[1]) and not (seen[1] & seen[2]) and len(seen[0] | seen[1] | seen[2]) == 48
    one = _store(lm, dataset=rows, shard_index=0, num_shards=1)
    assert {int(r[0]) // 16 for r in one.get_batch_tokens(48)} == set(range(48))


def test_checkpoint_restores_the_token_position(lm, tmp_path):
    s = _store(lm)
    s.get_batch_tokens()
    s.get_batch_tokens()
    s.save_to_checkpoint(tmp_path)
    nxt = s.get_batch_tokens()
    t = _store(lm)
    t.load_from_checkpoint(tmp_path)
    torch.testing.assert_close(t.get_batch_tokens(), nxt)


def test_reset_input_dataset_restarts_tokens(lm):
    s = _store(lm)
    first = s.get_batch_tokens()
    s.get_batch_tokens()
    s.reset_input_dataset()
    torch.testing.assert_close(s.get_batch_tokens(), first)


def test_from_sae_takes_hook_and_context_from_metadata(lm):
    sae = StandardSAE(StandardSAEConfig(d_in=32, d_sae=64, metadata=SAEMetadata(hook_name=HOOK, context_size=16)))
    s = ActivationsStore.from_sae(lm, sae, "synthetic:uniform:200:16")
    assert s.hook_name == HOOK and s.context_size == 16
    s = ActivationsStore.from_sae(lm, sae, "synthetic:uniform:200:16", context_size=8)
    assert s.context_size == 8


class _Tok:
    bos_token_id = 1
    eos_token_id = 2
    sep_token_id = None

    def encode(self, text):
        return [int(t) for t in text.split()]


@pytest.mark.parametrize("rows, expected", [
    # BOS-led rows longer than the context: each row is cut, nothing spills into the next context
    ([[1, 5, 6, 7, 8], [1, 9, 9, 9, 9]], [[1, 5, 6, 7], [1, 9, 9, 9]]),
    # rows pretokenized without BOS stay without it
    ([[5, 6, 7, 8, 3], [9, 4, 4, 4, 4]], [[5, 6, 7, 8], [9, 4, 4, 4]]),
])
def test_pretokenized_rows_are_cut_to_the_context(lm, rows, expected):
    with pytest.warns(RuntimeWarning, match="cut to its first 4 tokens"):
        s = _store(lm, dataset=[{"input_ids": r} for r in rows], context_size=4, store_batch_size_prompts=2,
                   prepend_bos=True, tokenizer=_Tok())
    assert s.get_batch_tokens().tolist() == expected
    assert s.n_dataset_processed == 2


def test_text_rows_are_packed_with_bos(lm):
    s = _store(lm, dataset=[{"text": "5 6 7"}, {"text": "8 9"}], context_size=4, store_batch_size_prompts=1,
               prepend_bos=True, tokenizer=_Tok(), sequence_separator_token=None)
    assert s.get_batch_tokens().tolist() == [[1, 5, 6, 7]]
