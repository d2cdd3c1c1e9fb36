"""Producer-LM kernels (RMSNorm, RoPE, gated activation) against fp32 PyTorch restatements, and a
hooked Llama-shaped LM forward with the native kernels against the same forward in PyTorch."""

import math

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dtype,one_plus", [(torch.bfloat16, False), (torch.bfloat16, True), (torch.float32, False)])
def test_rmsnorm(dtype, one_plus):
    from saelens_b200.ops import native

    torch.manual_seed(0)
    x = torch.randn(77, 4096, device="cuda").to(dtype)
    w = (torch.randn(4096, device="cuda") * 0.1 + (0 if one_plus else 1)).to(dtype)
    y = native().rmsnorm(x, w, 1e-6, one_plus)
    xf = x.float()
    ref = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + 1e-6) * ((1 + w.float()) if one_plus else w.float())
    tol = 1e-2 if dtype == torch.bfloat16 else 1e-5
    assert torch.allclose(y.float(), ref, atol=tol, rtol=tol)


def test_rope_in_place():
    from saelens_b200.models.lm.transformer import rotary_tables
    from saelens_b200.ops import native

    torch.manual_seed(0)
    B, S, H, d = 2, 33, 5, 128
    x = torch.randn(B, S, H, d, device="cuda").to(torch.bfloat16)
    cos, sin = rotary_tables(64, d, 10000.0, "cuda")
    y = x.clone()
    native().rope_(y, cos, sin, 0)
    x1, x2 = x[..., : d // 2].float(), x[..., d // 2 :].float()
    c, s = cos[:S][None, :, None, :], sin[:S][None, :, None, :]
    ref = torch.cat([x1 * c - x2 * s, x2 * c + x1 * s], -1)
    assert torch.allclose(y.float(), ref, atol=2e-2, rtol=2e-2)


@pytest.mark.parametrize("kind", [0, 1])
def test_gated_act(kind):
    from saelens_b200.ops import native

    torch.manual_seed(0)
    g = torch.randn(64, 1024, device="cuda").to(torch.bfloat16)
    u = torch.randn(64, 1024, device="cuda").to(torch.bfloat16)
    out = native().gated_act(g, u, kind)
    gf = g.float()
    act = gf * torch.sigmoid(gf) if kind == 0 else 0.5 * gf * (1 + torch.tanh(math.sqrt(2 / math.pi) * (gf + 0.044715 * gf**3)))
    assert torch.allclose(out.float(), act * u.float(), atol=2e-2, rtol=2e-2)


def test_llama_forward_native_matches_torch():
    from saelens_b200.models.lm import HookedLM, preset_config

    torch.manual_seed(0)
    cfg = preset_config("llama-3-8b", n_layers=2, d_model=256, n_heads=4, n_key_value_heads=2, d_mlp=512,
                        d_vocab=1000, n_ctx=64, dtype="bfloat16")
    lm = HookedLM(cfg).cuda()
    toks = torch.randint(0, 1000, (2, 32), device="cuda")
    with torch.no_grad():
        native_logits, cache = lm.run_with_cache(toks, names_filter="blocks.1.hook_resid_pre")
    with torch.enable_grad():
        torch_logits = lm(toks).detach()
    assert torch.allclose(native_logits.float(), torch_logits.float(), atol=0.15, rtol=0.05)
    assert cache["blocks.1.hook_resid_pre"].shape == (2, 32, 256)


@pytest.mark.parametrize("dtype,bias", [(torch.bfloat16, True), (torch.float32, True), (torch.bfloat16, False)])
def test_layernorm(dtype, bias):
    from saelens_b200.ops import native

    torch.manual_seed(1)
    x = (torch.randn(50, 768, device="cuda") * 3 + 1).to(dtype)
    w = (torch.randn(768, device="cuda") * 0.1 + 1).to(dtype)
    b = (torch.randn(768, device="cuda") * 0.1).to(dtype) if bias else None
    y = native().layernorm(x, w, b, 1e-5)
    ref = torch.nn.functional.layer_norm(x.float(), (768,), w.float(), b.float() if bias else None, 1e-5)
    tol = 2e-2 if dtype == torch.bfloat16 else 1e-5
    assert torch.allclose(y.float(), ref, atol=tol, rtol=tol)


def test_embed_gather_scale_and_positions():
    from saelens_b200.ops import native

    torch.manual_seed(2)
    table = torch.randn(1000, 256, device="cuda").to(torch.bfloat16)
    pos = torch.randn(64, 256, device="cuda").to(torch.bfloat16)
    toks = torch.randint(0, 1000, (3, 40), device="cuda")
    bad = torch.zeros(1, dtype=torch.int32, device="cuda")
    y = native().embed(toks, table, 1.0, pos, bad)
    assert torch.equal(y, table[toks] + pos[:40][None])
    y2 = native().embed(toks, table, 16.0, None, bad)
    assert torch.equal(y2, table[toks] * torch.tensor(16.0, dtype=torch.bfloat16, device="cuda"))
    assert int(bad) == 0
    toks[1, 5] = 1000
    y3 = native().embed(toks, table, 1.0, None, bad)
    assert int(bad) == 1 and torch.equal(y3[1, 5], torch.zeros_like(y3[1, 5]))


@pytest.mark.parametrize("preset, over", [
    ("gpt2", dict(n_layers=2, d_model=256, n_heads=4, d_mlp=1024, d_vocab=1001, n_ctx=300)),
    ("llama-3-8b", dict(n_layers=2, d_model=512, n_heads=8, n_key_value_heads=2, d_mlp=1408, d_vocab=2000,
                        n_ctx=300)),
    ("gemma-2-9b", dict(n_layers=2, d_model=512, n_heads=4, n_key_value_heads=2, d_head=256, d_mlp=1024,
                        d_vocab=2000, n_ctx=300, query_pre_attn_scalar=256.0)),
    ("qwen-14b", dict(n_layers=2, d_model=512, n_heads=4, n_key_value_heads=1, d_mlp=1000, d_vocab=2003,
                      n_ctx=300)),
])
def test_producer_families_native_against_torch_ops(preset, over):
    """The whole forward (embedding, norms, tcgen05 projections of any width, tcgen05 attention
    with GQA / soft-cap, gated MLP, unembedding) against the same model on PyTorch ops."""
    from saelens_b200.models.lm import transformer as T
    from saelens_b200.models.lm.transformer import HookedLM, preset_config

    torch.manual_seed(0)
    lm = HookedLM(preset_config(preset, dtype="bfloat16", **over)).cuda()
    toks = torch.randint(0, over["d_vocab"], (2, 257), device="cuda")
    # layer 0's q is cached (pre-rotation values kept: out-of-place RoPE), layer 1 rotates in place
    hooks = ["blocks.0.attn.hook_q", "blocks.1.hook_resid_pre", "blocks.1.attn.hook_z", "blocks.1.mlp.hook_pre",
             "blocks.1.hook_resid_post"]
    with torch.no_grad():
        logits, cache = lm.run_with_cache(toks, names_filter=hooks)
        T.FORCE_TORCH = True
        try:
            ref_logits, ref_cache = lm.run_with_cache(toks, names_filter=hooks)
        finally:
            T.FORCE_TORCH = False
    for h in hooks:
        a, b = cache[h].float(), ref_cache[h].float()
        rel = (a - b).norm() / b.norm()
        assert rel < 2e-2, (h, rel.item())
    rel = (logits.float() - ref_logits.float()).norm() / ref_logits.float().norm()
    assert rel < 3e-2, rel.item()
    assert logits.shape[-1] == over["d_vocab"]
