"""Shuffling buffer between the activation producer and the trainer
(behaviour of sae_lens/training/mixing_buffer.py:35-96).

Batches are concatenated until `buffer_size` rows are held; the buffer is permuted with a
dedicated generator, `mix_fraction` of it is kept for mixing with the next fill and the rest is
served in `batch_size` slices.  Dict batches (several hooks at once) are permuted jointly.
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


@torch.no_grad()
def mixing_buffer(buffer_size: int, batch_size: int, activations_loader: Iterator[Batch],
                  mix_fraction: float = 0.5, generator: torch.Generator | None = None) -> Iterator[Batch]:
    if buffer_size < batch_size:
        raise ValueError("Buffer size must be greater than or equal to batch size")
    if not 0 <= mix_fraction <= 1:
        raise ValueError("mix_fraction must be in [0, 1]")
    held: list[Batch] = []
    n_held = 0
    for batch in activations_loader:
        held.append(batch)
        n_held += _rows(batch)
        if n_held < buffer_size:
            continue
        buf = _cat(held)
        n = _rows(buf)
        if mix_fraction > 0:
            dev = next(iter(buf.values())).device if isinstance(buf, dict) else buf.device
            perm = torch.randperm(n, generator=generator, device="cpu").to(dev)
            buf = _take(buf, perm)
        keep = int(n * mix_fraction)
        serve = _take(buf, slice(keep, None))
        held = [_take(buf, slice(0, keep))] if keep > 0 else []
        n_held = keep
        n_serve = _rows(serve)
        for s in range(0, n_serve - batch_size + 1, batch_size):
            yield _take(serve, slice(s, s + batch_size))
        rem = n_serve % batch_size
        if rem:
            held.append(_take(serve, slice(n_serve - rem, None)))
            n_held += rem
    if n_held:
        buf = _cat(held)
        n = _rows(buf)
        for s in range(0, n - batch_size + 1, batch_size):
            yield _take(buf, slice(s, s + batch_size))
