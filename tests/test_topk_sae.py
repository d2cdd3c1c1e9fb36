"""TopK SAE math (behaviour of sae_lens/saes/topk_sae.py; cases follow tests/saes/test_topk_sae.py):
the aux-k loss against its formula, decoder-norm rescaling vs folding, sparse activations, and the
inference export."""

import pytest
import torch

from saelens_b200.models.sae import SAE, TrainStepInput
from saelens_b200.models.topk import TopKSAE, TopKSAEConfig, TopKTrainingSAE, TopKTrainingSAEConfig
from saelens_b200.registry import get_sae_class, get_sae_training_class


def _rand(sae, seed=0):
    torch.manual_seed(seed)
    with torch.no_grad():
        for p in sae.parameters():
            p.copy_(torch.randn_like(p) * 0.3)


def test_aux_loss_matches_formula():
    """Aux-k loss: the top-(d_in/2) pre-activations among dead latents (raw values, no ReLU)
    reconstruct the detached residual without b_dec; scaled by min(n_dead / k_aux, 1) and the
    coefficient."""
    torch.manual_seed(0)
    d_in, d_sae, k = 32, 96, 8
    sae = TopKTrainingSAE(TopKTrainingSAEConfig(d_in=d_in, d_sae=d_sae, k=k, rescale_acts_by_decoder_norm=False,
                                                aux_loss_coefficient=1.0))
    _rand(sae)
    x = torch.randn(50, d_in)
    dead = torch.zeros(d_sae, dtype=torch.bool)
    dead[::3] = True  # 32 dead latents
    out = sae.training_forward_pass(TrainStepInput(sae_in=x, coefficients={}, dead_neuron_mask=dead,
                                                   n_training_steps=0, is_logging_step=False))
    with torch.no_grad():
        pre = (x - sae.b_dec) @ sae.W_enc + sae.b_enc
        acts = torch.zeros_like(pre)
        top = pre.topk(k, dim=-1)
        acts.scatter_(1, top.indices, torch.relu(top.values))
        x_hat = acts @ sae.W_dec + sae.b_dec
        resid = x - x_hat
        k_aux = d_in // 2
        masked = torch.where(dead, pre, torch.full_like(pre, -torch.inf))
        t = masked.topk(k_aux, dim=-1)
        aux = torch.zeros_like(pre).scatter(1, t.indices, t.values)
        want = ((aux @ sae.W_dec - resid) ** 2).sum(-1).mean() * min(int(dead.sum()) / k_aux, 1.0)
    torch.testing.assert_close(out.losses["auxiliary_reconstruction_loss"].detach(), want, rtol=1e-4, atol=1e-5)


@pytest.mark.parametrize("rescale", [True, False])
def test_aux_loss_gives_b_dec_no_gradient(rescale):
    sae = TopKTrainingSAE(TopKTrainingSAEConfig(d_in=8, d_sae=12, k=4, rescale_acts_by_decoder_norm=rescale))
    _rand(sae)
    sae.b_dec.data = torch.randn(8) * 10.0
    x = torch.randn(10, 8)
    pre = x @ sae.W_enc + sae.b_enc
    if rescale:
        pre = pre * sae.W_dec.norm(dim=-1)
    out = sae.decode(sae.activation_fn(pre))
    sae.zero_grad()
    sae.calculate_topk_aux_loss(x, out, pre, torch.ones(12, dtype=torch.bool)).backward()
    assert sae.b_dec.grad is None or float(sae.b_dec.grad.abs().sum()) == pytest.approx(0.0, abs=1e-7)


@pytest.mark.parametrize("norm", ["constant_norm_rescale", "layer_norm"])
def test_aux_loss_rejects_activation_normalization(norm):
    sae = TopKTrainingSAE(TopKTrainingSAEConfig(d_in=8, d_sae=12, k=4, normalize_activations=norm))
    _rand(sae)
    x = torch.randn(10, 8)
    f, pre = sae.encode_with_hidden_pre(x)
    with pytest.raises(ValueError, match="does not support activation normalization"):
        sae.calculate_topk_aux_loss(x, sae.decode(f), pre, torch.ones(12, dtype=torch.bool))


def test_sparse_activations_config_is_respected():
    for flag in (True, False):
        sae = TopKTrainingSAE(TopKTrainingSAEConfig(d_in=8, d_sae=200, k=100, use_sparse_activations=flag))
        assert sae.activation_fn.use_sparse_activations is flag and sae.cfg.use_sparse_activations is flag


@pytest.mark.parametrize("training", [True, False])
def test_folding_decoder_norm_keeps_outputs_when_rescaling(training):
    cls, cfg_cls = get_sae_training_class("topk") if training else get_sae_class("topk")
    sae = cls(cfg_cls(k=2, d_in=5, d_sae=10, rescale_acts_by_decoder_norm=True))
    _rand(sae)
    x = torch.randn(300, 5)
    with torch.no_grad():
        f0 = sae.encode(x)
        y0 = sae.decode(f0)
        sae.fold_W_dec_norm()
        f1 = sae.encode(x)
        y1 = sae.decode(f1)
    torch.testing.assert_close(f1, f0, rtol=1e-2, atol=1e-4)
    torch.testing.assert_close(y1, y0, rtol=1e-2, atol=1e-4)
    torch.testing.assert_close(sae.W_dec.norm(dim=-1), torch.ones(10))


@pytest.mark.parametrize("training", [True, False])
def test_rescaling_equals_plain_topk_on_a_normalized_decoder(training):
    cls, cfg_cls = get_sae_training_class("topk") if training else get_sae_class("topk")
    a = cls(cfg_cls(k=2, d_in=5, d_sae=10, rescale_acts_by_decoder_norm=True))
    _rand(a)
    a.fold_W_dec_norm()
    b = cls(cfg_cls(k=2, d_in=5, d_sae=10, rescale_acts_by_decoder_norm=False))
    b.load_state_dict(a.state_dict())
    x = torch.randn(300, 5)
    with torch.no_grad():
        torch.testing.assert_close(a.encode(x), b.encode(x), rtol=1e-2, atol=1e-4)
        torch.testing.assert_close(a.decode(a.encode(x)), b.decode(b.encode(x)), rtol=1e-2, atol=1e-4)


@pytest.mark.parametrize("training", [True, False])
@pytest.mark.parametrize("case", ["k_full", "uniform_scale"])
def test_rescaling_changes_features_but_not_outputs(training, case):
    cls, cfg_cls = get_sae_training_class("topk") if training else get_sae_class("topk")
    k = 10 if case == "k_full" else 2
    a = cls(cfg_cls(k=k, d_in=5, d_sae=10, rescale_acts_by_decoder_norm=True))
    _rand(a)
    if case == "uniform_scale":
        a.fold_W_dec_norm()
        a.W_dec.data *= 0.5
    b = cls(cfg_cls(k=k, d_in=5, d_sae=10, rescale_acts_by_decoder_norm=False))
    b.load_state_dict(a.state_dict())
    x = torch.randn(300, 5)
    with torch.no_grad():
        assert not torch.allclose(a.encode(x), b.encode(x), rtol=1e-2)
        torch.testing.assert_close(a.decode(a.encode(x)), b.decode(b.encode(x)), rtol=1e-2, atol=1e-4)


@pytest.mark.parametrize("training", [True, False])
def test_fold_refused_without_rescaling(training):
    cls, cfg_cls = get_sae_training_class("topk") if training else get_sae_class("topk")
    with pytest.raises(NotImplementedError):
        cls(cfg_cls(d_in=5, d_sae=10, rescale_acts_by_decoder_norm=False)).fold_W_dec_norm()


@pytest.mark.parametrize("rescale", [True, False])
def test_training_sae_exports_equivalent_inference_sae(tmp_path, rescale):
    sae = TopKTrainingSAE(TopKTrainingSAEConfig(d_in=16, d_sae=48, k=4, rescale_acts_by_decoder_norm=rescale))
    _rand(sae)
    sae.save_inference_model(tmp_path)
    inf = SAE.load_from_disk(tmp_path)
    assert isinstance(inf, TopKSAE)
    x = torch.randn(40, 16)
    with torch.no_grad():
        torch.testing.assert_close(inf(x), sae.decode(sae.encode(x)), rtol=1e-4, atol=1e-5)


def test_inference_sae_save_load_roundtrip(tmp_path):
    sae = TopKSAE(TopKSAEConfig(d_in=16, d_sae=48, k=4))
    _rand(sae)
    sae.save_model(tmp_path)
    back = SAE.load_from_disk(tmp_path)
    x = torch.randn(10, 16)
    with torch.no_grad():
        torch.testing.assert_close(back(x), sae(x))
    assert back.cfg.k == 4


@pytest.mark.parametrize("ndim", [2, 3])
def test_sparse_activations_match_dense(ndim):
    cfg = TopKTrainingSAEConfig(d_in=16, d_sae=64, k=5)
    dense = TopKTrainingSAE(cfg)
    _rand(dense)
    sparse = TopKTrainingSAE(TopKTrainingSAEConfig(d_in=16, d_sae=64, k=5, use_sparse_activations=True))
    sparse.load_state_dict(dense.state_dict())
    x = torch.randn(*([3] * (ndim - 1)), 7, 16) if ndim == 3 else torch.randn(7, 16)
    with torch.no_grad():
        fd = dense.encode(x)
        fs = sparse.encode(x)
        fs_dense = fs.to_dense() if fs.is_sparse else fs
        torch.testing.assert_close(fs_dense, fd)
        torch.testing.assert_close(sparse.decode(fs), dense.decode(fd), rtol=1e-5, atol=1e-5)
        assert int((fd != 0).sum(-1).max()) <= 5
