"""BatchTopK activation and training SAE (behaviour of sae_lens/saes/batchtopk_sae.py; expected
values follow tests/saes/test_batchtopk_sae.py)."""

import pytest
import torch

from saelens_b200.models.batchtopk import BatchTopK, BatchTopKTrainingSAE, BatchTopKTrainingSAEConfig
from saelens_b200.models.jumprelu import JumpReLUSAE
from saelens_b200.models.sae import SAE, TrainStepInput


def _step(x):
    return TrainStepInput(sae_in=x, coefficients={}, dead_neuron_mask=None, n_training_steps=0,
                          is_logging_step=False)


@pytest.mark.parametrize("k,x,expected", [
    (2, [[1.0, -2.0, 3.0, -4.0], [-5.0, 6.0, -7.0, 8.0]], [[1.0, 0.0, 3.0, 0.0], [0.0, 6.0, 0.0, 8.0]]),
    (2, [[1.0, 2.0, 3.0, 4.0], [-5.0, -6.0, 0.5, -8.0]], [[1.0, 2.0, 3.0, 4.0], [0.0, 0.0, 0.0, 0.0]]),
    (1.5, [[1.0, -2.0, 3.0, -4.0], [-5.0, 6.0, -7.0, 8.0]], [[0.0, 0.0, 3.0, 0.0], [0.0, 6.0, 0.0, 8.0]]),
    (2, [[-1.0, 2.0, -3.0, -4.0], [5.0, -6.0, -7.0, -8.0]], [[0.0, 2.0, 0.0, 0.0], [5.0, 0.0, 0.0, 0.0]]),
])
def test_batch_topk_selects_over_the_whole_batch(k, x, expected):
    out = BatchTopK(k=k)(torch.tensor(x))
    torch.testing.assert_close(out, torch.tensor(expected))
    assert (out >= 0).all()


@pytest.mark.parametrize("shape", [(20,), (10, 20), (4, 8, 20), (2, 3, 4, 20)])
def test_average_l0_equals_k_for_any_leading_shape(shape):
    torch.manual_seed(0)
    out = BatchTopK(k=5)(torch.randn(*shape) + 2.0)
    assert out.shape == shape
    assert (out != 0).sum().item() / torch.Size(shape[:-1]).numel() == pytest.approx(5)


def test_config_accepts_float_k():
    assert BatchTopKTrainingSAEConfig(d_in=8, d_sae=16, k=2.5).k == 2.5


def test_training_step_updates_threshold_and_reports_it():
    torch.manual_seed(0)
    sae = BatchTopKTrainingSAE(BatchTopKTrainingSAEConfig(d_in=16, d_sae=32, k=4))
    sae.topk_threshold = torch.tensor(0.0)
    sae.b_enc.data = torch.randn(32) + 10
    with torch.no_grad():
        out = sae.training_forward_pass(_step(torch.randn(4, 16)))
    assert float(sae.topk_threshold) != 0.0
    assert out.metrics["topk_threshold"] == sae.topk_threshold


def test_threshold_is_ema_of_min_positive_kept_activation():
    torch.manual_seed(1)
    lr = 0.25
    sae = BatchTopKTrainingSAE(BatchTopKTrainingSAEConfig(d_in=16, d_sae=32, k=4, topk_threshold_lr=lr,
                                                          rescale_acts_by_decoder_norm=False))
    sae.topk_threshold = torch.tensor(0.3, dtype=torch.float64)
    x = torch.randn(8, 16)
    with torch.no_grad():
        f, _ = sae.encode_with_hidden_pre(x)
        before = float(sae.topk_threshold)
        sae.training_forward_pass(_step(x))
    m = float(f[f > 0].min())
    assert float(sae.topk_threshold) == pytest.approx((1 - lr) * before + lr * m, rel=1e-5)


def test_inference_config_and_state_dict_are_jumprelu():
    sae = BatchTopKTrainingSAE(BatchTopKTrainingSAEConfig(d_in=8, d_sae=16, k=2))
    d = sae.cfg.get_inference_sae_cfg_dict()
    assert d["architecture"] == "jumprelu" and d["d_in"] == 8 and d["d_sae"] == 16
    assert "topk_threshold_lr" not in d
    sae.topk_threshold = torch.tensor(0.5)
    sd = sae.state_dict()
    sae.process_state_dict_for_saving_inference(sd)
    assert "topk_threshold" not in sd
    torch.testing.assert_close(sd["threshold"], torch.full_like(sae.b_enc, 0.5))


@pytest.mark.parametrize("rescale", [True, False])
def test_inference_jumprelu_reproduces_thresholded_training_sae(tmp_path, rescale):
    torch.manual_seed(0)
    sae = BatchTopKTrainingSAE(BatchTopKTrainingSAEConfig(d_in=16, d_sae=48, k=4,
                                                          rescale_acts_by_decoder_norm=rescale))
    with torch.no_grad():
        for p in sae.parameters():
            p.copy_(torch.randn_like(p) * 0.3)
    sae.topk_threshold = torch.tensor(0.2, dtype=torch.float64)
    sae.save_inference_model(tmp_path)
    inf = SAE.load_from_disk(tmp_path)
    assert isinstance(inf, JumpReLUSAE)
    x = torch.randn(30, 16)
    with torch.no_grad():
        pre = (x - sae.b_dec) @ sae.W_enc + sae.b_enc
        if rescale:
            pre = pre * sae.W_dec.norm(dim=-1)
        acts = torch.where(pre > 0.2, pre, torch.zeros_like(pre))
        if rescale:
            acts = acts / sae.W_dec.norm(dim=-1)
        want = acts @ sae.W_dec + sae.b_dec
        torch.testing.assert_close(inf(x), want, rtol=1e-4, atol=1e-5)


@pytest.mark.parametrize("case", ["fold", "normalized", "k_full", "uniform_scale"])
def test_decoder_norm_rescaling_equivalences(case):
    torch.manual_seed(0)
    k = 10 if case == "k_full" else 2
    a = BatchTopKTrainingSAE(BatchTopKTrainingSAEConfig(d_in=5, d_sae=10, k=k, rescale_acts_by_decoder_norm=True))
    with torch.no_grad():
        for p in a.parameters():
            p.copy_(torch.randn_like(p))
    x = torch.randn(300, 5)
    with torch.no_grad():
        if case == "fold":
            f0 = a.encode(x)
            y0 = a.decode(f0)
            a.fold_W_dec_norm()
            torch.testing.assert_close(a.encode(x), f0, rtol=1e-2, atol=1e-4)
            torch.testing.assert_close(a.decode(a.encode(x)), y0, rtol=1e-2, atol=1e-4)
            return
        if case in ("normalized", "uniform_scale"):
            a.fold_W_dec_norm()
        if case == "uniform_scale":
            a.W_dec.data *= 0.5
        b = BatchTopKTrainingSAE(BatchTopKTrainingSAEConfig(d_in=5, d_sae=10, k=k,
                                                            rescale_acts_by_decoder_norm=False))
        b.load_state_dict(a.state_dict())
        fa, fb = a.encode(x), b.encode(x)
        if case == "normalized":
            torch.testing.assert_close(fa, fb, rtol=1e-2, atol=1e-4)
        else:
            assert not torch.allclose(fa, fb, rtol=1e-2)
        torch.testing.assert_close(a.decode(fa), b.decode(fb), rtol=1e-2, atol=1e-4)
