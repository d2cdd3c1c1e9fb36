"""Numerics of each sm_100a kernel against a plain PyTorch fp32 restatement of the same op."""

import pytest
import torch

pytestmark = pytest.mark.gpu


def _ops():
    from saelens_b200 import ops

    assert ops.available(), "native extension must load on a GPU box"
    return ops


@pytest.mark.parametrize(
    "M,N,K",
    [(128, 256, 64), (256, 512, 128), (300, 1024, 768), (1000, 2048, 4096), (17, 256, 256)],
)
def test_gemm_tn_matches_fp32(M, N, K):
    ops = _ops()
    a = torch.randn(M, K, device="cuda").to(torch.bfloat16)
    b = torch.randn(N, K, device="cuda").to(torch.bfloat16)
    out, _ = ops.gemm_tn(a, b)
    ref = a.float() @ b.float().T
    torch.cuda.synchronize()
    err = (out.float() - ref).abs().max().item()
    tol = 1e-2 * ref.abs().max().item() + 1e-3
    assert err <= tol, f"max err {err} > {tol}"


@pytest.mark.parametrize("M,N,K", [(300, 1000, 1000), (513, 50257, 64), (128, 40, 24), (1024, 2003, 776)])
def test_gemm_ragged_width_and_depth(M, N, K):
    """Any N (partial last 256-column tile, masked epilogue) and K a multiple of 8 (the ragged last
    k-block reads zeros past K), with a bias, on both the single-CTA and the CTA-pair kernel."""
    ops = _ops()
    a = torch.randn(M, K, device="cuda").to(torch.bfloat16)
    b = torch.randn(N, K, device="cuda").to(torch.bfloat16)
    bias = torch.randn(N, device="cuda")
    guard = 7.0
    buf = torch.full((M, (N + 7) // 8 * 8 + 8), guard, dtype=torch.bfloat16, device="cuda")
    out = buf[:, :N]
    ops.gemm_tn(a, b, bias=bias, out=out)
    ref = a.float() @ b.float().T + bias
    torch.cuda.synchronize()
    assert (out.float() - ref).abs().max().item() <= 1e-2 * ref.abs().max().item() + 1e-3
    assert (buf[:, N:] == guard).all(), "columns past N were written"
    auto, _ = ops.gemm_tn(a, b, bias=bias)
    assert auto.shape == (M, N) and torch.equal(auto, out)


def test_gemm_epilogue_bias_scale_relu_chunkmax():
    ops = _ops()
    M, N, K = 384, 768, 512
    a = torch.randn(M, K, device="cuda").to(torch.bfloat16)
    b = torch.randn(N, K, device="cuda").to(torch.bfloat16)
    bias = torch.randn(N, device="cuda")
    scale = torch.rand(N, device="cuda") + 0.5
    out, cmax = ops.gemm_tn(a, b, bias=bias, scale=scale, relu=True, chunk_max=True)
    ref = torch.relu((a.float() @ b.float().T + bias) * scale)
    torch.cuda.synchronize()
    assert (out.float() - ref).abs().max().item() <= 1e-2 * ref.abs().max().item() + 1e-3
    ref_cmax = out.float().view(M, N // 32, 32).amax(-1)
    assert torch.equal(cmax.float(), ref_cmax)


def test_gemm_many_tiles_persistent():
    # more tiles than SMs so every CTA loops over several tiles and both TMEM buffers
    ops = _ops()
    M, N, K = 2048, 4096, 256
    a = torch.randn(M, K, device="cuda").to(torch.bfloat16)
    b = torch.randn(N, K, device="cuda").to(torch.bfloat16)
    out, _ = ops.gemm_tn(a, b)
    ref = a.float() @ b.float().T
    torch.cuda.synchronize()
    assert (out.float() - ref).abs().max().item() <= 1e-2 * ref.abs().max().item() + 1e-3
    out2, _ = ops.gemm_tn(a, b, max_ctas=7)
    assert torch.equal(out, out2)


@pytest.mark.parametrize("M,N,K", [(512, 1024, 256), (300, 50257, 64), (1000, 2003, 776)])
def test_pair_gemm_tma_stores_equal_row_stores(monkeypatch, M, N, K):
    """The CTA-pair kernel's TMA tile stores (staging tile, 128-byte swizzle, clipped at M and N)
    write exactly what the per-thread row stores write, and nothing past column N."""
    ops = _ops()
    a = torch.randn(M, K, device="cuda").to(torch.bfloat16)
    b = torch.randn(N, K, device="cuda").to(torch.bfloat16)
    bias = torch.randn(N, device="cuda")
    outs = {}
    for tma in ("1", "0"):
        monkeypatch.setenv("SAELENS_B200_GEMM_TMA_STORE", tma)
        buf = torch.full((M, (N + 7) // 8 * 8 + 8), 7.0, dtype=torch.bfloat16, device="cuda")
        cm = torch.empty(M, N // 32, dtype=torch.bfloat16, device="cuda") if N % 32 == 0 else None
        ops.native().gemm_tn_bf16(a, b, bias, None, True, buf[:, :N], cm, ops.StatusWord("cuda").tensor, 0)
        torch.cuda.synchronize()
        assert (buf[:, N:] == 7.0).all(), "columns past N were written"
        outs[tma] = (buf.clone(), cm)
    assert torch.equal(outs["1"][0], outs["0"][0])
    if outs["1"][1] is not None:
        assert torch.equal(outs["1"][1], outs["0"][1])


def _check_topk(h, vals, idx, k):
    M, N = h.shape
    hf = h.float()
    ref_v, _ = torch.topk(hf, k, dim=-1)
    kth = ref_v[:, -1:]
    # every selected index is distinct, valid, carries its own value, and is >= the k-th value
    assert (idx >= 0).all() and (idx < N).all()
    s = torch.sort(idx.long(), dim=-1).values
    assert (s[:, 1:] != s[:, :-1]).all()
    got = torch.gather(hf, 1, idx.long())
    assert torch.equal(got, vals)
    assert (vals >= kth).all()
    # same multiset of values as torch.topk
    assert torch.equal(torch.sort(vals, dim=-1).values, torch.sort(ref_v, dim=-1).values)


@pytest.mark.parametrize("M,N,k", [(8, 256, 16), (64, 4096, 64), (32, 32768, 128), (4, 1024, 1024)])
def test_row_topk_exact(M, N, k):
    ops = _ops()
    h = torch.randn(M, N, device="cuda").to(torch.bfloat16)
    cmax = h.float().view(M, N // 32, 32).amax(-1).to(torch.bfloat16)
    vals, idx = ops.row_topk(h, cmax, k)
    torch.cuda.synchronize()
    _check_topk(h, vals, idx, k)


def test_row_topk_ties_and_overflow_fallback():
    ops = _ops()
    M, N, k = 4, 65536, 64
    h = torch.zeros(M, N, device="cuda", dtype=torch.bfloat16)  # all ties -> fallback path
    h[1, 100:200] = 1.0
    cmax = h.float().view(M, N // 32, 32).amax(-1).to(torch.bfloat16)
    vals, idx = ops.row_topk(h, cmax, k)
    torch.cuda.synchronize()
    _check_topk(h, vals, idx, k)
    # ties are broken by the smaller index
    assert torch.equal(torch.sort(idx[0]).values.cpu(), torch.arange(k, dtype=torch.int32))
    assert torch.equal(torch.sort(idx[1]).values.cpu(), torch.arange(100, 100 + k, dtype=torch.int32))


def test_decode_mse_matches_dense():
    ops = _ops()
    M, N, D, k = 64, 2048, 768, 32
    W = (torch.randn(N, D, device="cuda") * 0.05).to(torch.bfloat16)
    vals = torch.randn(M, k, device="cuda")
    idx = torch.stack([torch.randperm(N, device="cuda")[:k] for _ in range(M)]).int()
    idx[0, 5] = -1
    inv = torch.rand(N, device="cuda") + 0.5
    bias = torch.randn(D, device="cuda") * 0.1
    x = torch.randn(M, D, device="cuda").to(torch.bfloat16)
    res = ops.decode_mse(vals, idx, W, x, inv_scale=inv, bias=bias, grad_coef=2.0 / M, want_bsum=True)
    F = torch.zeros(M, N, device="cuda")
    live = idx >= 0
    coef = torch.relu(vals) * inv[idx.clamp(min=0).long()]
    F.scatter_(1, idx.clamp(min=0).long(), torch.where(live, coef, torch.zeros_like(coef)))
    xh = F @ W.float() + bias
    err = xh - x.float()
    torch.cuda.synchronize()
    assert torch.allclose(res["out"].float(), xh, atol=2e-2, rtol=2e-2)
    assert torch.allclose(res["loss_row"], err.pow(2).sum(-1), rtol=1e-3, atol=1e-3)
    assert torch.allclose(res["dxhat"].float(), err * 2.0 / M, atol=1e-4, rtol=2e-2)
    assert torch.allclose(res["bsum"], (err * 2.0 / M).sum(0), atol=1e-3, rtol=2e-2)
