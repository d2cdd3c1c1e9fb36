"""ActivationScaler (behaviour of sae_lens/training/activation_scaler.py; cases follow
tests/training/test_activation_scaler.py)."""

import pytest
import torch

from saelens_b200.training.activation_scaler import ActivationScaler


def test_identity_without_factor():
    s = ActivationScaler()
    x = torch.randn(4, 8)
    assert torch.equal(s.scale(x), x) and torch.equal(s.unscale(x), x) and torch.equal(s(x), x)


@pytest.mark.parametrize("f", [0.5, 1.0, 2.0, 10.0])
def test_scale_unscale_roundtrip(f):
    s = ActivationScaler(scaling_factor=f)
    x = torch.randn(32, 64)
    torch.testing.assert_close(s.scale(x), x * f)
    torch.testing.assert_close(s(x), x * f)
    torch.testing.assert_close(s.unscale(s.scale(x)), x, rtol=1e-6, atol=1e-6)


def test_zero_negative_and_shapes():
    s = ActivationScaler(scaling_factor=3.0)
    assert torch.equal(s.scale(torch.zeros(10, 20)), torch.zeros(10, 20))
    torch.testing.assert_close(s.scale(torch.tensor([[-1.0, 2.0], [-3.0, 4.0]])),
                               torch.tensor([[-3.0, 6.0], [-9.0, 12.0]]))
    for shape in [(1, 1), (10, 64), (4, 16, 32)]:
        assert s.unscale(s.scale(torch.randn(*shape))).shape == shape


def test_mean_norm_over_batches():
    batches = iter([torch.tensor([[3.0, 4.0]]), torch.tensor([[6.0, 8.0]]), torch.tensor([[0.0, 0.0]]),
                    torch.tensor([[1.0, 0.0]]), torch.tensor([[0.0, 2.0]])])
    assert ActivationScaler()._calculate_mean_norm(batches, n_batches_for_norm_estimate=5) == pytest.approx(18 / 5)


def test_estimate_scaling_factor():
    def const(d, v):
        while True:
            yield torch.full((10, d), v)

    s = ActivationScaler()
    s.estimate_scaling_factor(d_in=64, data_provider=const(64, 2.0), n_batches_for_norm_estimate=10)
    assert s.scaling_factor == pytest.approx(0.5)  # sqrt(64) / 16


def test_save_and_load(tmp_path):
    s = ActivationScaler(scaling_factor=1.25)
    with pytest.raises(ValueError, match=".json"):
        s.save(str(tmp_path / "scaler.txt"))
    s.save(str(tmp_path / "scaler.json"))
    t = ActivationScaler()
    t.load(tmp_path / "scaler.json")
    assert t.scaling_factor == 1.25
