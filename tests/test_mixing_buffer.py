"""Mixing buffer (behaviour of sae_lens/training/mixing_buffer.py; cases follow
tests/training/test_mixing_buffer.py)."""

from collections.abc import Iterator

import pytest
import torch

from saelens_b200.training.mixing_buffer import mixing_buffer


def test_batch_size_holds_despite_loader_size_changes():
    acts = [torch.randn(19, 8), torch.randn(15, 8)]  # 34 rows -> 8 batches of 4
    out = list(mixing_buffer(buffer_size=16, batch_size=4, activations_loader=iter(acts)))
    assert len(out) == 8 and all(b.shape == (4, 8) for b in out)


def test_mixes_and_never_duplicates():
    acts = [torch.arange(30), torch.arange(30, 60), torch.arange(60, 120)]
    b = next(mixing_buffer(buffer_size=100, batch_size=50, activations_loader=iter(acts)))
    assert b.shape == (50,)
    assert not torch.equal(b, torch.arange(50))
    assert len(torch.unique(b)) == 50


def test_empty_loader_yields_nothing():
    assert not list(mixing_buffer(buffer_size=16, batch_size=4, activations_loader=iter([])))


def test_buffer_smaller_than_batch_raises():
    with pytest.raises(ValueError):
        next(mixing_buffer(buffer_size=4, batch_size=8, activations_loader=iter([torch.randn(8, 4)])))


@pytest.mark.parametrize("mix_fraction", [-0.1, 1.5])
def test_invalid_mix_fraction_raises(mix_fraction):
    with pytest.raises(ValueError, match="mix_fraction must be in"):
        next(mixing_buffer(buffer_size=16, batch_size=4, activations_loader=iter([torch.randn(16, 8)]),
                           mix_fraction=mix_fraction))


def test_dtype_is_kept():
    acts = [torch.randn(4, 8, dtype=torch.float64) for _ in range(2)]
    assert all(b.dtype == torch.float64 for b in mixing_buffer(16, 4, iter(acts)))


def test_total_batches_independent_of_mix_fraction():
    for frac in (0.2, 0.7):
        acts = [torch.randn(100, 8), torch.randn(100, 8)]
        assert len(list(mixing_buffer(100, 10, iter(acts), mix_fraction=frac))) == 20


def test_zero_mix_fraction_is_passthrough():
    out = torch.cat(list(mixing_buffer(100, 10, iter([torch.arange(100)]), mix_fraction=0)))
    assert torch.equal(out, torch.arange(100))


def test_every_row_served_exactly_once():
    acts = [torch.arange(i * 37, (i + 1) * 37) for i in range(10)]
    out = torch.cat(list(mixing_buffer(64, 8, iter(acts), mix_fraction=0.5)))
    assert len(out) % 8 == 0 and len(out) > 370 - 8  # whole batches; under one batch left over
    assert len(torch.unique(out)) == len(out)


def test_dict_batches_share_one_permutation():
    acts = [{"a": torch.arange(16).unsqueeze(-1), "b": (torch.arange(16) + 100).unsqueeze(-1)}]
    out = list(mixing_buffer(16, 8, iter(acts), mix_fraction=0.5))
    assert len(out) == 2
    for b in out:
        assert torch.equal(b["b"].squeeze(-1), b["a"].squeeze(-1) + 100)


def test_generator_decouples_from_global_rng():
    acts = [torch.arange(16), torch.arange(16, 32)]
    out1 = list(mixing_buffer(16, 8, iter(acts), 0.5, generator=torch.Generator().manual_seed(1234)))
    torch.rand(1000)
    out2 = list(mixing_buffer(16, 8, iter(acts), 0.5, generator=torch.Generator().manual_seed(1234)))
    assert len(out1) == len(out2) and all(torch.equal(a, b) for a, b in zip(out1, out2))


def test_observed_mix_fraction_matches_target():
    target, size = 0.7, 10_000

    def rows():
        for i in range(100_000):
            yield torch.tensor([i])

    fracs = []
    for i, b in enumerate(mixing_buffer(size, 1000, rows(), mix_fraction=target)):
        if i > 10:
            old = b.max().item() - (1 - target) * size
            fracs.append(float((b < old).sum()) / len(b))
    assert sum(fracs) / len(fracs) == pytest.approx(target, abs=0.03)


@pytest.mark.parametrize("mix_fraction", [0.9, 1.0])
def test_storage_stays_bounded_with_high_mix_fraction(mix_fraction):
    size, bs = 100, 10
    served = [0]
    worst = [0]

    def loader() -> Iterator[torch.Tensor]:
        for i in range(20):
            worst[0] = max(worst[0], i * size - served[0] * bs)
            yield torch.randn(size, 8)

    for _ in mixing_buffer(size, bs, loader(), mix_fraction=mix_fraction):
        served[0] += 1
    assert worst[0] <= 2 * size
