"""Producer LMs: hook coverage, stop-at-layer, and logit parity with transformers' own
implementations on tiny random-init configs (the HF model is the oracle)."""

import pytest
import torch

from saelens_b200.models.lm import HookedLM, preset_config
from saelens_b200.models.lm.hf import HookedProxyLM, hooked_lm_from_hf

transformers = pytest.importorskip("transformers")


def _tiny_llama(model_type="llama"):
    if model_type == "qwen2":
        cfg = transformers.Qwen2Config(vocab_size=300, hidden_size=64, intermediate_size=128, num_hidden_layers=2,
                                       num_attention_heads=4, num_key_value_heads=2, max_position_embeddings=64)
        return transformers.Qwen2ForCausalLM(cfg)
    cfg = transformers.LlamaConfig(vocab_size=300, hidden_size=64, intermediate_size=128, num_hidden_layers=2,
                                   num_attention_heads=4, num_key_value_heads=2, max_position_embeddings=64)
    return transformers.LlamaForCausalLM(cfg)


@pytest.mark.parametrize("model_type", ["llama", "qwen2"])
def test_converted_llama_family_matches_hf(model_type):
    torch.manual_seed(0)
    hf = _tiny_llama(model_type).eval()
    lm = hooked_lm_from_hf(hf).eval()
    toks = torch.randint(0, 300, (2, 12))
    with torch.no_grad():
        ref = hf(input_ids=toks).logits
        got = lm(toks)
    assert torch.allclose(got, ref, atol=1e-4, rtol=1e-4)


def test_converted_gpt2_matches_hf():
    torch.manual_seed(0)
    hf = transformers.GPT2LMHeadModel(transformers.GPT2Config(vocab_size=200, n_embd=64, n_layer=2, n_head=4,
                                                              n_positions=32)).eval()
    lm = hooked_lm_from_hf(hf).eval()
    toks = torch.randint(0, 200, (2, 10))
    with torch.no_grad():
        assert torch.allclose(lm(toks), hf(input_ids=toks).logits, atol=1e-4, rtol=1e-4)


def test_resid_hooks_match_hf_hidden_states():
    torch.manual_seed(1)
    hf = _tiny_llama().eval()
    lm = hooked_lm_from_hf(hf).eval()
    toks = torch.randint(0, 300, (1, 9))
    with torch.no_grad():
        hs = hf(input_ids=toks, output_hidden_states=True).hidden_states
        _, cache = lm.run_with_cache(toks, names_filter=lambda n: "resid_pre" in n)
    assert torch.allclose(cache["blocks.1.hook_resid_pre"], hs[1], atol=1e-5)


def test_stop_at_layer_and_hook_editing():
    lm = HookedLM(preset_config("gpt2", n_layers=3, d_model=64, n_heads=4, d_mlp=128, d_vocab=100, dtype="float32"))
    toks = torch.randint(0, 100, (2, 8))
    out, cache = lm.run_with_cache(toks, stop_at_layer=2, names_filter="blocks.1.hook_resid_post")
    assert torch.equal(out, cache["blocks.1.hook_resid_post"])
    base = lm(toks)
    edited = lm.run_with_hooks(toks, fwd_hooks=[("blocks.0.hook_mlp_out", lambda t, hook: t * 0)])
    assert not torch.allclose(base, edited)
    assert torch.allclose(lm(toks), base)  # hooks are removed afterwards


def test_hooked_proxy_lm_stops_early():
    hf = _tiny_llama().eval()
    proxy = HookedProxyLM(hf)
    toks = torch.randint(0, 300, (1, 5))
    out, cache = proxy.run_with_cache(toks, names_filter="model.layers.0", stop_at_layer=1)
    assert out is None and cache["model.layers.0"].shape == (1, 5, 64)
    assert "model.layers.1" not in proxy.run_with_cache(toks, names_filter="model.layers.1", stop_at_layer=1)[1]
