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
