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


def test_hooked_proxy_lm_return_types_and_option_checks():
    import pytest

    from saelens_b200.models.lm.hf import _extract_logits_from_output

    hf = _tiny_llama().eval()
    proxy = HookedProxyLM(hf)
    toks = torch.randint(0, 300, (2, 6))
    with torch.no_grad():
        logits = proxy(toks)
        both_logits, loss = proxy(toks, return_type="both")
        torch.testing.assert_close(both_logits, logits)
        lp = torch.log_softmax(logits[:, :-1].float(), -1)
        want = -lp.gather(-1, toks[:, 1:].unsqueeze(-1)).mean()
        torch.testing.assert_close(loss.float(), want, rtol=1e-4, atol=1e-4)
        for bad in ("loss", "activations"):
            with pytest.raises(NotImplementedError, match="Only return_type supported is"):
                proxy(toks, return_type=bad)
        with pytest.raises(NotImplementedError, match="stop_at_layer is not supported for return_type='both'"):
            proxy(toks, return_type="both", stop_at_layer=1)
        out_tuple = hf(input_ids=toks, return_dict=False)
        torch.testing.assert_close(_extract_logits_from_output(out_tuple), logits)
    with pytest.raises(ValueError, match="Unsupported model output type"):
        _extract_logits_from_output("not an output")

    class _Obj:
        def __init__(self, lg):
            self.logits = lg

    assert _extract_logits_from_output(_Obj(None)) is None
    torch.testing.assert_close(_extract_logits_from_output(_Obj(logits)), logits)


def test_hooked_proxy_to_tokens_options_and_unknown_model_class():
    import pytest

    from saelens_b200.models.lm.load_model import load_model

    proxy = HookedProxyLM(_tiny_llama(), tokenizer=lambda t, **kw: {"input_ids": torch.tensor([[5, 6]] * len(t))})
    assert proxy.to_tokens("hi").tolist() == [[5, 6]]
    for kw, msg in [({"prepend_bos": True}, "prepend_bos=False"), ({"prepend_bos": None}, "prepend_bos=False"),
                    ({"padding_side": "left"}, "padding_side=None"), ({"truncate": True}, "truncate=False"),
                    ({"move_to_device": True}, "move_to_device=False")]:
        with pytest.raises(ValueError, match=f"Only works with {msg}"):
            proxy.to_tokens("hi", **kw)
    with pytest.raises(ValueError, match="Unknown model class: FakeModelClass"):
        load_model("FakeModelClass", "some-model", device="cpu")


def test_load_model_vllm_class_name_gives_the_native_producer():
    from saelens_b200.models.lm.load_model import load_model
    from saelens_b200.models.lm.transformer import HookedLM

    lm = load_model("VLLMModel", "gpt2", device="cpu",
                    model_from_pretrained_kwargs={"gpu_memory_utilization": 0.5, "max_model_len": 128,
                                                  "enforce_eager": True, "n_layers": 1, "dtype": "float32"})
    assert isinstance(lm, HookedLM) and lm.cfg.n_layers == 1


def test_load_model_hooked_mamba_needs_mamba_lens():
    import pytest

    from saelens_b200.models.lm.load_model import load_model

    with pytest.raises(ValueError, match="mamba-lens"):
        load_model("HookedMamba", "state-spaces/mamba-130m")
