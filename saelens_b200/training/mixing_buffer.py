"""Shuffling buffer between the activation producer and the trainer
(behaviour of sae_lens/training/mixing_buffer.py:35-96).

Batches are concatenated until `buffer_size` rows are held; the buffer is permuted with a
dedicated generator, `mix_fraction * buffer_size` rows are kept for mixing with the next fill and
the rest is served in `batch_size` slices.  Dict batches (several hooks at once) are permuted
jointly.  The fill / permute / serve steps match the reference's so that a given generator seed
yields the same batches.
"""

from __future__ import annotations

from collections.abc import Iterator

import torch

Batch = torch.Tensor | dict[str, torch.Tensor]


def _rows(b: Batch) -> int:
    return next(iter(b.values())).shape[0] if isinstance(b, dict) else b.shape[0]


def _cat(parts: list[Batch]) -> Batch:
    if isinstance(parts[0], dict):
        return {k: torch.cat([p[k] for p in parts], dim=0) for k in parts[0]}  # type: ignore[index]
    return torch.cat(parts, dim=0)  # type: ignore[arg-type]


def _take(b: Batch, idx: torch.Tensor | slice) -> Batch:
    if isinstance(b, dict):
        return {k: v[idx] for k, v in b.items()}
    return b[idx]


def _permute(parts: list[Batch], perm: torch.Tensor) -> Batch:
    """`cat(parts)[perm]`.  On CUDA one native pass gathers from the last part and the rows
    before it (`ops.gather_rows`), so the concatenated buffer is never written first."""
    first = parts[0]
    t0 = next(iter(first.values())) if isinstance(first, dict) else first
    if not t0.is_cuda:
        return _take(_cat(parts), perm)
    from saelens_b200 import ops

    head = parts[0] if len(parts) <= 2 else _cat(parts[:-1])
    tail = parts[-1] if len(parts) >= 2 else None
    if isinstance(head, dict):
        return {k: ops.gather_rows(v, None if tail is None else tail[k], perm)  # type: ignore[index]
                for k, v in head.items()}
    return ops.gather_rows(head, tail, perm)  # type: ignore[arg-type]


@torch.no_grad()
def mixing_buffer(buffer_size: int, batch_size: int, activations_loader: Iterator[Batch],
                  mix_fraction: float = 0.5, generator: torch.Generator | None = None) -> Iterator[Batch]:
    """Whenever at least `buffer_size` rows are held: permute them (CPU `randperm` on
    `generator`, so a seed gives the same stream on any device), serve whole batches from the
    front and hold the last `int(buffer_size * mix_fraction)` rows (at least one batch is served
    per fill, so even `mix_fraction=1` keeps the held rows bounded).  With `mix_fraction=0` rows
    are served in arrival order.  Leftover rows are served unshuffled at the end, whole batches
    only."""
    if buffer_size < batch_size:
        raise ValueError("Buffer size must be greater than or equal to batch size")
    if not 0 <= mix_fraction <= 1:
        raise ValueError("mix_fraction must be in [0, 1]")
    keep = int(buffer_size * mix_fraction)
    parts: list[Batch] = []  # held rows first, then the batches received since the last fill
    n = 0
    for batch in activations_loader:
        parts.append(batch)
        n += _rows(batch)
        if n < buffer_size:
            continue
        if mix_fraction > 0:
            dev = next(iter(batch.values())).device if isinstance(batch, dict) else batch.device
            held = _permute(parts, torch.randperm(n, generator=generator).to(dev))
        else:
            held = parts[0] if len(parts) == 1 else _cat(parts)
        n_batches = max(1, (n - keep) // batch_size)
        cut = n_batches * batch_size
        serve, rest = _take(held, slice(0, cut)), _take(held, slice(cut, None))
        parts, n = ([rest] if n > cut else []), n - cut
        for i in range(n_batches):
            yield _take(serve, slice(i * batch_size, (i + 1) * batch_size))
    if parts:
        held = parts[0] if len(parts) == 1 else _cat(parts)
        for i in range(_rows(held) // batch_size):
            yield _take(held, slice(i * batch_size, (i + 1) * batch_size))
