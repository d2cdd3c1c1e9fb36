"""Packing of token sequences into contexts: the same token stream as
sae_lens/tokenization_and_batching.py (expected outputs follow the cases of
tests/test_tokenization_and_batching.py)."""

from itertools import islice

import pytest
import torch

from saelens_b200.training.tokenization_and_batching import concat_and_batch_sequences

A19 = torch.arange(19)
S4 = [A19[:3], A19[3:10], A19[10:17], A19[17:]]
S5 = [A19[:3], A19[3:8], A19[8:11], A19[11:17], A19[17:]]


def _run(seqs, **kw):
    return [b.tolist() for b in concat_and_batch_sequences(tokens_iterator=iter(seqs), context_size=5, **kw)]


def test_plain_packing_and_final_partial_dropped():
    a20 = torch.arange(20)
    assert _run([a20[:3], a20[3:10], a20[10:17], a20[17:]]) == a20.reshape(4, 5).tolist()
    assert _run(S4) == A19[:15].reshape(3, 5).tolist()


CASES = [
    (S4, dict(begin_batch_token_id=999),
     [[999, 0, 1, 2, 3], [999, 4, 5, 6, 7], [999, 8, 9, 10, 11], [999, 12, 13, 14, 15]]),
    (S4, dict(begin_batch_token_id=999, disable_concat_sequences=True), [[999, 3, 4, 5, 6], [999, 10, 11, 12, 13]]),
    (S4, dict(disable_concat_sequences=True), [[3, 4, 5, 6, 7], [10, 11, 12, 13, 14]]),
    (S4, dict(begin_sequence_token_id=998),
     [[998, 0, 1, 2, 998], [3, 4, 5, 6, 7], [8, 9, 998, 10, 11], [12, 13, 14, 15, 16]]),
    (S4, dict(begin_sequence_token_id=999, disable_concat_sequences=True), [[999, 3, 4, 5, 6], [999, 10, 11, 12, 13]]),
    (S4, dict(begin_batch_token_id=999, begin_sequence_token_id=999, disable_concat_sequences=True),
     [[999, 3, 4, 5, 6], [999, 10, 11, 12, 13]]),
    (S4, dict(begin_batch_token_id=999, begin_sequence_token_id=888, disable_concat_sequences=True),
     [[888, 3, 4, 5, 6], [888, 10, 11, 12, 13]]),
    (S4, dict(sequence_separator_token_id=997),
     [[0, 1, 2, 997, 3], [4, 5, 6, 7, 8], [9, 997, 10, 11, 12], [13, 14, 15, 16, 997]]),
    (S5, dict(sequence_separator_token_id=997, begin_sequence_token_id=998, begin_batch_token_id=999),
     [[999, 998, 0, 1, 2], [999, 998, 3, 4, 5], [999, 6, 7, 997, 998], [999, 8, 9, 10, 997],
      [999, 11, 12, 13, 14], [999, 15, 16, 997, 998]]),
    (S5, dict(sequence_separator_token_id=999, begin_sequence_token_id=999, begin_batch_token_id=999),
     [[999, 0, 1, 2, 999], [999, 3, 4, 5, 6], [999, 7, 999, 8, 9], [999, 10, 999, 11, 12], [999, 13, 14, 15, 16]]),
]


@pytest.mark.parametrize("seqs,kw,expected", CASES)
def test_special_token_rules(seqs, kw, expected):
    assert _run(seqs, **kw) == expected


def test_extremely_long_sample_is_streamed():
    out = list(islice(concat_and_batch_sequences(iter([torch.arange(10_000_000)]), 5, begin_sequence_token_id=999,
                                                 begin_batch_token_id=999), 50_000))
    assert len(out) == 50_000
    assert all(b.shape == (5,) and int(b[0]) == 999 for b in out)


def test_empty_sequences_with_disabled_concat():
    seqs = [torch.tensor([], dtype=torch.long), torch.arange(10), torch.tensor([], dtype=torch.long), torch.arange(5, 15)]
    assert _run(seqs, begin_batch_token_id=999, disable_concat_sequences=True) == [[999, 0, 1, 2, 3], [999, 5, 6, 7, 8]]
    assert _run(seqs[:2], begin_sequence_token_id=999, disable_concat_sequences=True) == [[999, 0, 1, 2, 3]]


def test_rejects_2d_tokens():
    with pytest.raises(ValueError, match="1D"):
        list(concat_and_batch_sequences(iter([torch.zeros(2, 3, dtype=torch.long)]), 5))
