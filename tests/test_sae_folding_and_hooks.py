"""Decoder-norm folding, device / dtype moves and SAE hooks for every architecture (behaviour of
sae_lens/saes/*; cases follow tests/saes/test_standard_sae.py)."""

import pytest
import torch

from saelens_b200.models.sae import SAE, TrainingSAE, _disable_hooks
from saelens_b200.registry import get_sae_class, get_sae_training_class

INF = ["standard", "gated", "jumprelu", "topk"]
TRAIN = ["standard", "gated", "jumprelu", "topk", "batchtopk", "matryoshka_batchtopk", "matching_pursuit"]


def _inf_cfg(arch, d_in=8, d_sae=16, **kw):
    extra = {"k": 3} if arch == "topk" else {}
    extra.update(kw)
    return get_sae_class(arch)[1](d_in=d_in, d_sae=d_sae, **extra)


def _train_cfg(arch, d_in=8, d_sae=16):
    extra = {}
    if arch in ("topk", "batchtopk", "matryoshka_batchtopk"):
        extra["k"] = 3
    if arch == "matryoshka_batchtopk":
        extra["matryoshka_widths"] = [4, d_sae]
    return get_sae_training_class(arch)[1](d_in=d_in, d_sae=d_sae, **extra)


def _rand(sae, seed=0):
    torch.manual_seed(seed)
    with torch.no_grad():
        for p in sae.parameters():
            p.copy_(torch.rand_like(p))


@pytest.mark.parametrize("arch", ["standard", "gated", "jumprelu"])
def test_fold_W_dec_norm_keeps_outputs(arch):
    sae = SAE.from_dict(_inf_cfg(arch).to_dict())
    _rand(sae)
    x = torch.randn(20, 8)
    with torch.no_grad():
        y0 = sae(x)
        f0 = sae.encode(x)
        norms = sae.W_dec.norm(dim=-1)
        sae.fold_W_dec_norm()
        torch.testing.assert_close(sae.W_dec.norm(dim=-1), torch.ones(16))
        torch.testing.assert_close(sae(x), y0, rtol=1e-4, atol=1e-4)
        torch.testing.assert_close(sae.encode(x), f0 * norms, rtol=1e-4, atol=1e-4)


@pytest.mark.parametrize("arch", INF)
def test_fold_W_dec_norm_zero_rows_make_no_nan(arch):
    sae = SAE.from_dict(_inf_cfg(arch, rescale_acts_by_decoder_norm=True) .to_dict() if arch == "topk"
                        else _inf_cfg(arch).to_dict())
    _rand(sae)
    sae.W_dec.data[:5] = 0.0
    sae.fold_W_dec_norm()
    for n, p in sae.named_parameters():
        assert torch.isfinite(p).all(), n


@pytest.mark.parametrize("arch", TRAIN)
def test_training_fold_W_dec_norm_zero_rows_make_no_nan(arch):
    sae = TrainingSAE.from_dict(_train_cfg(arch).to_dict())
    _rand(sae)
    sae.W_dec.data[:5] = 0.0
    if arch == "matching_pursuit":
        with pytest.raises(NotImplementedError):
            sae.fold_W_dec_norm()
        return
    sae.fold_W_dec_norm()
    for n, p in sae.named_parameters():
        assert torch.isfinite(p).all(), n


def test_topk_inference_fold_without_rescaling_refused():
    sae = SAE.from_dict(_inf_cfg("topk", rescale_acts_by_decoder_norm=False).to_dict())
    with pytest.raises(NotImplementedError):
        sae.fold_W_dec_norm()


def test_to_moves_dtype_and_returns_self():
    sae = SAE.from_dict(_inf_cfg("standard").to_dict())
    assert sae.to(torch.float64) is sae
    assert sae.W_enc.dtype == torch.float64 and sae.dtype == torch.float64
    sae.to("cpu", torch.float32)
    assert sae.W_dec.dtype == torch.float32 and sae.device == torch.device("cpu")
    sae.to(dtype=torch.bfloat16)
    assert sae.b_enc.dtype == torch.bfloat16
    sae.to(torch.zeros(1, dtype=torch.float32))
    assert sae.W_enc.dtype == torch.float32
    sae.to()
    assert sae.W_enc.dtype == torch.float32


def test_get_name():
    sae = SAE.from_dict(_inf_cfg("standard").to_dict())
    sae.cfg.metadata.model_name = "gpt2"
    sae.cfg.metadata.hook_name = "blocks.0.hook_resid_pre"
    assert sae.get_name() == "sae_gpt2_blocks.0.hook_resid_pre_16"


def test_disable_hooks_stops_and_restores_hooks():
    sae = SAE.from_dict(_inf_cfg("standard", d_in=2, d_sae=3).to_dict())
    x = torch.randn(10, 2)
    out0, cache0 = sae.run_with_cache(x)
    with _disable_hooks(sae):
        out1, cache1 = sae.run_with_cache(x)
    out2, cache2 = sae.run_with_cache(x)
    torch.testing.assert_close(out0, out1)
    torch.testing.assert_close(out0, out2)
    assert set(cache1) == set()
    assert set(cache0) == set(cache2) and all(torch.equal(cache0[k], cache2[k]) for k in cache0)


@pytest.mark.parametrize("arch", ["standard", "gated", "jumprelu"])
def test_error_term_unchanged_by_hook_interventions(arch):
    sae = SAE.from_dict(_inf_cfg(arch, d_in=32, d_sae=64).to_dict())
    _rand(sae)
    sae._use_error_term = True
    x = torch.randn(10, 32)
    out0, cache0 = sae.run_with_cache(x)

    def ablate(acts, hook):
        acts[:, :] = 20
        return acts

    with sae.hooks(fwd_hooks=[("hook_sae_acts_post", ablate)]):
        out1, cache1 = sae.run_with_cache(x)
    assert not torch.allclose(out0, out1, rtol=1e-2)
    assert torch.all(cache1["hook_sae_acts_post"] == 20)
    torch.testing.assert_close(cache0["hook_sae_error"], cache1["hook_sae_error"], rtol=1e-4, atol=1e-5)


@pytest.mark.parametrize("mode", ["constant_norm_rescale", "layer_norm", "none"])
def test_run_time_normalization_is_undone_on_output(mode):
    sae = SAE.from_dict(_inf_cfg("standard", normalize_activations=mode).to_dict())
    _rand(sae)
    x = torch.randn(6, 8) * 5 + 3
    with torch.no_grad():
        y1 = sae(x)
        y2 = sae(x * 2.0)
    if mode in ("constant_norm_rescale", "layer_norm"):
        # the input scale is removed before encoding and restored on the output
        torch.testing.assert_close(sae.encode(x * 2.0), sae.encode(x), rtol=1e-4, atol=1e-4)
        torch.testing.assert_close(y2, 2.0 * y1, rtol=1e-4, atol=1e-4)
    else:
        assert not torch.allclose(sae.encode(x * 2.0), sae.encode(x))
