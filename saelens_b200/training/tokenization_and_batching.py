"""Pack tokenized sequences into fixed-length training contexts.

Packing rules (the same token stream as sae_lens/tokenization_and_batching.py, so activations
line up token for token with the reference):
* every context starts with `begin_batch_token_id` (unless it already starts with it);
* every sequence starts with `begin_sequence_token_id` (unless it already does);
* consecutive sequences inside one context are joined by `sequence_separator_token_id`
  (unless the next sequence already starts with it);
* a sequence that overflows a context continues in the next one, which gets only the batch
  token; prefix tokens that no longer fit are dropped;
* with `disable_concat_sequences`, sequences are not joined: each is truncated to the context
  (after prepending the sequence token) and shorter ones are skipped.
"""

from __future__ import annotations

from collections.abc import Iterator

import torch


def _starts_with(seq: list[int], pos: int, tok: int | None) -> bool:
    return tok is not None and pos < len(seq) and seq[pos] == tok


@torch.no_grad()
def concat_and_batch_sequences(tokens_iterator: Iterator[torch.Tensor], context_size: int,
                               begin_batch_token_id: int | None = None, begin_sequence_token_id: int | None = None,
                               sequence_separator_token_id: int | None = None,
                               disable_concat_sequences: bool = False) -> Iterator[torch.Tensor]:
    if disable_concat_sequences:
        bos = begin_sequence_token_id if begin_sequence_token_id is not None else begin_batch_token_id
        for t in tokens_iterator:
            seq = t.tolist()
            if bos is not None and len(seq) >= context_size - 1 and (not seq or seq[0] != bos):
                seq = [bos] + seq[: context_size - 1]
            if len(seq) >= context_size:
                yield torch.tensor(seq[:context_size], dtype=torch.long)
        return
    ctx: list[int] | None = None
    for t in tokens_iterator:
        if t.dim() != 1:
            raise ValueError(f"tokens.shape should be 1D but was {tuple(t.shape)}")
        seq = t.tolist()
        off = 0
        first_piece = True
        while off < len(seq):
            prefix: list[int] = []
            head = seq[off]
            if first_piece and begin_sequence_token_id is not None and head != begin_sequence_token_id:
                prefix.append(begin_sequence_token_id)
                head = begin_sequence_token_id
            if ctx is None:
                if begin_batch_token_id is not None and head != begin_batch_token_id:
                    prefix.insert(0, begin_batch_token_id)
                need = max(context_size - len(prefix), 0)
                ctx = prefix[:context_size] + seq[off : off + need]
                off += need
            else:
                if sequence_separator_token_id is not None and head != sequence_separator_token_id:
                    prefix.insert(0, sequence_separator_token_id)
                room = max(context_size - len(ctx), 0)
                need = max(room - len(prefix), 0)
                ctx = ctx + prefix[:room] + seq[off : off + need]
                off += need
            first_piece = False
            if len(ctx) == context_size:
                yield torch.tensor(ctx, dtype=torch.long)
                ctx = None
