"""tcgen05 prefill attention (`ops.attention`) against an fp32 PyTorch softmax(q k^T * scale) v of
the same bf16 inputs: causal and full, grouped-query heads, head dims 64 / 128 / 256, Gemma-2's
logit soft-cap, sequence lengths that are not a multiple of the 128-row tile, and q / k / v given
as strided views of one fused projection output."""

import math

import pytest
import torch

pytestmark = pytest.mark.gpu


def _oracle(q, k, v, scale, softcap=None, causal=True):
    B, S, H, D = q.shape
    KV = k.shape[2]
    qf = q.float().transpose(1, 2)                                   # [B, H, S, D]
    kf = k.float().transpose(1, 2).repeat_interleave(H // KV, dim=1)
    vf = v.float().transpose(1, 2).repeat_interleave(H // KV, dim=1)
    s = qf @ kf.transpose(-1, -2) * scale
    if softcap:
        s = softcap * torch.tanh(s / softcap)
    if causal:
        mask = torch.ones(S, S, dtype=torch.bool, device=q.device).tril()
        s = s.masked_fill(~mask, float("-inf"))
    return (torch.softmax(s, dim=-1) @ vf).transpose(1, 2)           # [B, S, H, D]


def _inputs(B, S, H, KV, D, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    mk = lambda h: torch.randn(B, S, h, D, generator=g, device="cuda").to(torch.bfloat16)  # noqa: E731
    return mk(H), mk(KV), mk(KV)


def _check(out, ref):
    err = (out.float() - ref).abs()
    # bf16 output rounding (2^-9 relative) plus bf16 probabilities in the P.V product
    assert err.max().item() <= 3e-2, err.max().item()
    assert err.mean().item() <= 3e-3, err.mean().item()


@pytest.mark.parametrize("S", [128, 1024, 2048])
def test_causal_gqa_32_8_head_dim_128(S):
    from saelens_b200 import ops

    q, k, v = _inputs(1, S, 32, 8, 128, seed=S)
    scale = 1 / math.sqrt(128)
    _check(ops.attention(q, k, v, scale), _oracle(q, k, v, scale))


@pytest.mark.parametrize("B, S, H, KV, D", [
    (2, 100, 12, 12, 64),     # GPT-2 heads, a partial tile
    (3, 300, 8, 2, 128),      # several batches, partial last tile, group of 4
    (1, 257, 16, 8, 256),     # Gemma-2 head size (64-row K/V tiles)
])
def test_causal_shapes(B, S, H, KV, D):
    from saelens_b200 import ops

    q, k, v = _inputs(B, S, H, KV, D, seed=B * S + D)
    scale = 1 / math.sqrt(D)
    _check(ops.attention(q, k, v, scale), _oracle(q, k, v, scale))


def test_gemma2_softcap_and_query_scalar():
    from saelens_b200 import ops

    q, k, v = _inputs(1, 512, 16, 8, 256, seed=5)
    q = (q.float() * 4).to(torch.bfloat16)  # large logits, so the soft-cap matters
    scale = 1 / math.sqrt(256.0)
    out = ops.attention(q, k, v, scale, softcap=50.0)
    ref = _oracle(q, k, v, scale, softcap=50.0)
    _check(out, ref)
    assert (ref - _oracle(q, k, v, scale)).abs().max().item() > 0.05  # the cap changed the result


def test_full_attention_without_mask():
    from saelens_b200 import ops

    q, k, v = _inputs(2, 200, 4, 4, 64, seed=9)
    _check(ops.attention(q, k, v, 0.125, causal=False), _oracle(q, k, v, 0.125, causal=False))


def test_views_of_a_fused_projection_and_repeated_calls():
    from saelens_b200 import ops

    B, S, H, KV, D = 2, 384, 8, 2, 128
    g = torch.Generator(device="cuda").manual_seed(3)
    qkv = torch.randn(B, S, (H + 2 * KV) * D, generator=g, device="cuda").to(torch.bfloat16)
    q = qkv[..., : H * D].view(B, S, H, D)
    k = qkv[..., H * D : (H + KV) * D].view(B, S, KV, D)
    v = qkv[..., (H + KV) * D :].view(B, S, KV, D)
    assert not q.is_contiguous()
    ref = _oracle(q, k, v, 0.1)
    first = ops.attention(q, k, v, 0.1)
    _check(first, ref)
    assert torch.equal(ops.attention(q, k, v, 0.1), first)  # deterministic


def test_rejects_unsupported_head_dim():
    from saelens_b200 import ops

    q, k, v = _inputs(1, 128, 2, 2, 96, seed=1)
    with pytest.raises(ValueError, match="head dim must be 64, 128 or 256"):
        ops.attention(q, k, v, 0.1)


@pytest.mark.parametrize("D, softcap", [(64, None), (128, None), (256, 30.0)])
def test_four_and_eight_softmax_warps_agree(monkeypatch, D, softcap):
    """The whole-row (4 softmax warps) and half-row (8 warps, exchanged row maxima and sums)
    kernels both match the fp32 oracle, on a length with a partial last tile."""
    from saelens_b200 import ops

    q, k, v = _inputs(2, 333, 8, 4, D, seed=D)
    scale = 1 / math.sqrt(D)
    ref = _oracle(q, k, v, scale, softcap=softcap)
    outs = {}
    for w in ("4", "8"):
        monkeypatch.setenv("SAELENS_B200_ATTN_WARPS", w)
        outs[w] = ops.attention(q, k, v, scale, softcap=softcap)
        _check(outs[w], ref)
    assert (outs["4"].float() - outs["8"].float()).abs().max().item() <= 2e-2
