"""HookedSAETransformer: splicing SAEs and transcoders into the hooked LM (behaviour of
sae_lens/analysis/hooked_sae_transformer.py; cases follow tests/test_hooked_sae_transformer.py)."""

import logging

import pytest
import torch

from saelens_b200.analysis.hooked_sae_transformer import HookedSAETransformer, _get_module, _SAEWrapper
from saelens_b200.models.lm.transformer import preset_config
from saelens_b200.models.standard import StandardSAE, StandardSAEConfig
from saelens_b200.models.transcoder import Transcoder, TranscoderConfig
from saelens_b200.utils.hooks import HookPoint

D = 32
ACTS = ["blocks.0.hook_resid_pre", "blocks.0.hook_mlp_out", "blocks.1.hook_resid_post", "blocks.0.attn.hook_z"]


@pytest.fixture
def model():
    torch.manual_seed(0)
    m = HookedSAETransformer(preset_config("gpt2", n_layers=2, d_model=D, n_heads=4, d_mlp=64, d_vocab=97,
                                           n_ctx=16, dtype="float32"))
    m.eval()
    return m


@pytest.fixture
def tokens():
    return torch.randint(0, 97, (2, 8))


def _sae(act: str, seed: int = 1) -> StandardSAE:
    torch.manual_seed(seed)
    d_in = D
    cfg = StandardSAEConfig(d_in=d_in, d_sae=2 * d_in)
    if act.endswith("hook_z"):
        cfg = StandardSAEConfig(d_in=d_in, d_sae=2 * d_in, reshape_activations="hook_z")
    sae = StandardSAE(cfg)
    with torch.no_grad():  # nonzero biases so the spliced model differs from the clean one
        sae.b_enc.normal_(0, 0.1)
        sae.b_dec.normal_(0, 0.1)
    sae.cfg.metadata.hook_name = act
    if act.endswith("hook_z"):
        sae.turn_on_forward_pass_hook_z_reshaping()
    return sae


def _transcoder(seed: int = 2) -> Transcoder:
    torch.manual_seed(seed)
    tc = Transcoder(TranscoderConfig(d_in=D, d_sae=2 * D, d_out=D, apply_b_dec_to_input=False))
    tc.cfg.metadata.hook_name = "blocks.0.mlp.hook_in"
    tc.cfg.metadata.hook_name_out = "blocks.0.hook_mlp_out"
    return tc


def test_no_saes_matches_original_and_saes_change_output(model, tokens):
    with torch.no_grad():
        ref = model(tokens)
        assert torch.equal(model.run_with_saes(tokens, saes=[]), ref)
        spliced = model.run_with_saes(tokens, saes=[_sae(a) for a in ACTS])
    assert not torch.allclose(spliced, ref, atol=1e-4)
    assert model.acts_to_saes == {}
    with torch.no_grad():
        assert torch.equal(model(tokens), ref)  # fully restored


def test_add_sae_replaces_hook_point_and_unwraps(model):
    sae = _sae(ACTS[1])
    model.add_sae(sae)
    wrapper = _get_module(model, ACTS[1])
    assert isinstance(wrapper, _SAEWrapper) and wrapper.sae is sae
    assert model.acts_to_saes == {ACTS[1]: sae}
    # the SAE's own hooks are addressable under the LM hook name
    assert f"{ACTS[1]}.hook_sae_acts_post" in model.hook_dict
    model.reset_saes()
    assert isinstance(_get_module(model, ACTS[1]), HookPoint)
    assert f"{ACTS[1]}.hook_sae_acts_post" not in model.hook_dict


def test_add_sae_warns_for_invalid_hook(model, caplog):
    sae = _sae("invalid.hook.name")
    with caplog.at_level(logging.WARNING):
        model.add_sae(sae)
    assert "No hook found for invalid.hook.name" in caplog.text
    assert len(model._acts_to_saes) == 0


def test_reset_sae_warns_for_unattached(model, caplog):
    with caplog.at_level(logging.WARNING):
        model._reset_sae("blocks.0.hook_mlp_out")
    assert "No SAE is attached to blocks.0.hook_mlp_out" in caplog.text


def test_add_sae_overwrites_and_reset_replaces(model):
    a, b = _sae(ACTS[0], 1), _sae(ACTS[0], 2)
    model.add_sae(a)
    model.add_sae(b)
    assert len(model._acts_to_saes) == 1 and model._acts_to_saes[ACTS[0]].sae is b
    model._reset_sae(ACTS[0], _SAEWrapper(a))
    assert len(model._acts_to_saes) == 1 and _get_module(model, ACTS[0]).sae is a
    model._reset_sae(ACTS[0])
    assert len(model._acts_to_saes) == 0 and isinstance(_get_module(model, ACTS[0]), HookPoint)


def test_reset_saes_specific_names(model):
    saes = [_sae(a, i) for i, a in enumerate(ACTS[:3])]
    for s in saes:
        model.add_sae(s)
    model.reset_saes(ACTS[:2])
    assert list(model.acts_to_saes) == [ACTS[2]]
    model.reset_saes()
    assert model.acts_to_saes == {}


def test_context_manager_restores_previous_saes(model, tokens):
    prev = [_sae(a, 10 + i) for i, a in enumerate(ACTS[:3])]
    for s in prev:
        model.add_sae(s)
    with torch.no_grad():
        before = model(tokens)
    new = [_sae(a, 20 + i) for i, a in enumerate(ACTS[:3])]
    with model.saes(saes=new):
        for a, s in zip(ACTS[:3], new):
            assert model.acts_to_saes[a] is s
        with torch.no_grad():
            model(tokens)
    assert [model.acts_to_saes[a] for a in ACTS[:3]] == prev
    with torch.no_grad():
        assert torch.equal(model(tokens), before)
    model.reset_saes()


def test_context_manager_restores_after_exception(model):
    sae = _sae(ACTS[1])
    original = sae.use_error_term
    with pytest.raises(RuntimeError):
        with model.saes(saes=[sae], use_error_term=True):
            assert _get_module(model, ACTS[1]).use_error_term is True
            raise RuntimeError("inside")
    assert sae.use_error_term == original
    assert len(model._acts_to_saes) == 0


def test_use_error_term_settings(model):
    sae = _sae(ACTS[1])
    for flag, want in [(True, True), (False, False), (None, False)]:
        model.add_sae(sae, use_error_term=flag)
        assert _get_module(model, ACTS[1]).use_error_term is want
    model.reset_saes()
    sae._use_error_term = True
    model.add_sae(sae, use_error_term=None)
    assert _get_module(model, ACTS[1]).use_error_term is True
    model.add_sae(sae, use_error_term=False)  # explicit False overrides the SAE's setting
    assert _get_module(model, ACTS[1]).use_error_term is False
    model.reset_saes()
    sae._use_error_term = False


@pytest.mark.parametrize("act", ACTS)
def test_error_term_reproduces_clean_model(model, tokens, act):
    with torch.no_grad():
        ref = model(tokens)
        out = model.run_with_saes(tokens, saes=[_sae(act)], use_error_term=True)
        out_cache, cache = model.run_with_cache_with_saes(tokens, saes=[_sae(act)], use_error_term=True)
    torch.testing.assert_close(out, ref, atol=1e-4, rtol=1e-4)
    torch.testing.assert_close(out_cache, ref, atol=1e-4, rtol=1e-4)
    assert f"{act}.hook_sae_error" in cache and f"{act}.hook_sae_acts_post" in cache


def test_run_with_cache_with_saes_records_sae_hooks(model, tokens):
    sae = _sae(ACTS[2])
    with torch.no_grad():
        _, cache = model.run_with_cache_with_saes(tokens, saes=[sae])
        feats = sae.encode(cache[ACTS[2]])
    torch.testing.assert_close(cache[f"{ACTS[2]}.hook_sae_input"], cache[ACTS[2]])
    torch.testing.assert_close(cache[f"{ACTS[2]}.hook_sae_acts_post"], feats)
    assert cache[f"{ACTS[2]}.hook_sae_output"].shape == (2, 8, D)
    assert model.acts_to_saes == {}


def test_hook_z_sae_keeps_head_shape(model, tokens):
    sae = _sae(ACTS[3])
    with torch.no_grad():
        ref = model(tokens)
        out, cache = model.run_with_cache_with_saes(tokens, saes=[sae], use_error_term=False)
    assert not torch.allclose(out, ref, atol=1e-4)
    assert cache[f"{ACTS[3]}.hook_sae_output"].shape == (2, 8, 4, D // 4)


def test_run_with_hooks_with_saes(model, tokens):
    sae = _sae(ACTS[1])
    seen = []

    def grab(t, hook):
        seen.append(hook.name)

    with torch.no_grad():
        model.run_with_hooks_with_saes(tokens, saes=[sae], fwd_hooks=[(f"{ACTS[1]}.hook_sae_acts_post", grab)])
    assert seen == [f"{ACTS[1]}.hook_sae_acts_post"]
    assert model.acts_to_saes == {}
    assert not model.hook_dict[ACTS[1]]._fwd_handles


def test_mlp_hook_in_is_cached(model, tokens):
    with torch.no_grad():
        _, cache = model.run_with_cache(tokens)
    for n in range(2):
        assert cache[f"blocks.{n}.mlp.hook_in"].shape == (2, 8, D)


def test_error_term_unchanged_when_latents_ablated(model, tokens):
    sae = _sae(ACTS[1])
    with torch.no_grad():
        out0, cache0 = model.run_with_cache_with_saes(tokens, saes=[sae], use_error_term=True)
    assert cache0[f"{ACTS[1]}.hook_sae_acts_post"].abs().sum() > 0
    model.add_sae(sae, use_error_term=True)
    with torch.no_grad(), model.hooks(fwd_hooks=[(f"{ACTS[1]}.hook_sae_acts_post", lambda t, hook: t * 0)]):
        out1, cache1 = model.run_with_cache(tokens)
    model.reset_saes()
    assert cache1[f"{ACTS[1]}.hook_sae_acts_post"].abs().sum() == 0
    torch.testing.assert_close(cache1[f"{ACTS[1]}.hook_sae_error"], cache0[f"{ACTS[1]}.hook_sae_error"])
    assert not torch.allclose(out1, out0, atol=1e-5)


def test_transcoder_splices_and_matches_manual(model, tokens):
    tc = _transcoder()
    with torch.no_grad():
        ref, clean = model.run_with_cache(tokens)
        out, cache = model.run_with_cache_with_saes(tokens, saes=[tc])
        expected = tc.decode(tc.encode(cache["blocks.0.mlp.hook_in"]))
    assert not torch.allclose(out, ref, atol=1e-4)
    torch.testing.assert_close(cache["blocks.0.hook_mlp_out.hook_sae_output"], expected, atol=1e-5, rtol=1e-5)
    # with the error term the output is the clean one
    with torch.no_grad():
        out_err = model.run_with_saes(tokens, saes=[tc], use_error_term=True)
    torch.testing.assert_close(out_err, ref, atol=1e-4, rtol=1e-4)
    assert model.acts_to_saes == {}
    assert not model.hook_dict["blocks.0.mlp.hook_in"]._fwd_handles  # the input grab is gone
    # a user's permanent hook on the input hook survives the transcoder's removal
    model.add_hook("blocks.0.mlp.hook_in", lambda t, hook: None, is_permanent=True)
    model.run_with_saes(tokens, saes=[tc])
    assert len(model.hook_dict["blocks.0.mlp.hook_in"]._fwd_handles) == 1
    model.reset_hooks(including_permanent=True)


def test_mixed_sae_and_transcoder_gradients_flow(model, tokens):
    tc, sae = _transcoder(), _sae(ACTS[2])
    model.add_sae(tc)
    model.add_sae(sae)
    model(tokens).sum().backward()
    for m in (tc, sae):
        assert m.W_enc.grad is not None and m.W_enc.grad.abs().sum() > 0
        assert m.W_dec.grad is not None and m.W_dec.grad.abs().sum() > 0
    model.reset_saes()
