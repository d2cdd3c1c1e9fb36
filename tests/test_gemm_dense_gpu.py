"""The dense-step tcgen05 GEMM (`ops.gemm_dense`) against fp32 PyTorch restatements: K-major and
MN-major operands (no transposes in memory), ragged sizes, and every epilogue mode the dense SAE
steps use (JumpReLU forward / backward with the rectangle-window threshold gradient, fused MSE and
dL/dx_hat, rank-1 correction, gated pre-activations, column sums and counts)."""

import pytest
import torch

pytestmark = pytest.mark.gpu


def _bf(*shape, scale=1.0, seed=0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    return (torch.randn(*shape, generator=g, device="cuda") * scale).to(torch.bfloat16)


def _close(got, ref, rel=1e-2):
    err = (got.float() - ref).abs().max().item()
    assert err <= rel * ref.abs().max().item() + 1e-2, err


@pytest.mark.parametrize("a_mn, b_mn", [(False, False), (False, True), (True, False), (True, True)])
@pytest.mark.parametrize("M, N, K", [(256, 512, 256), (304, 1000, 200), (1024, 2048, 1024)])
def test_layouts_and_ragged_sizes(a_mn, b_mn, M, N, K):
    from saelens_b200 import ops

    a = _bf(K, M, seed=1) if a_mn else _bf(M, K, seed=1)
    b = _bf(K, N, seed=2) if b_mn else _bf(N, K, seed=2)
    A = a.float().T if a_mn else a.float()
    B = b.float() if b_mn else b.float().T
    bias = torch.randn(N, device="cuda")
    out = ops.gemm_dense(a, b, a_mn=a_mn, b_mn=b_mn, bias=bias)
    _close(out, A @ B + bias)


def test_jumprelu_forward_outputs_pre_acts_counts_and_l0():
    from saelens_b200 import ops

    M, N, K = 384, 768, 512
    x, w = _bf(M, K, seed=3), _bf(N, K, scale=0.05, seed=4)
    bias = torch.randn(N, device="cuda") * 0.1
    thr = torch.rand(N, device="cuda") * 0.5
    pre = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
    cnt = torch.zeros(N, device="cuda")
    nnz = torch.zeros(1, dtype=torch.int64, device="cuda")
    acts = ops.gemm_dense(x, w, out2=pre, bias=bias, thr=thr, colcnt=cnt, nnz=nnz)
    ref_pre = x.float() @ w.float().T + bias
    _close(pre, ref_pre)
    pre_f = pre.float()
    ref_acts = torch.where(pre_f > thr, pre_f, torch.zeros_like(pre_f))
    assert torch.equal(acts.float(), ref_acts)
    assert torch.equal(cnt, (acts != 0).float().sum(0))
    assert int(nnz) == int((acts != 0).sum())


def test_decode_residual_mse_and_bias_gradient_sums():
    from saelens_b200 import ops

    B, D, N = 512, 384, 2048
    f = torch.relu(_bf(B, N, seed=5)).to(torch.bfloat16)
    w_dec = _bf(N, D, scale=0.05, seed=6)               # stored [d_sae, d_in]: MN-major B
    b_dec = torch.randn(D, device="cuda") * 0.1
    x = _bf(B, D, seed=7)
    recon = torch.empty(B, D, dtype=torch.bfloat16, device="cuda")
    loss = torch.zeros(1, device="cuda")
    bsum = torch.zeros(D, device="cuda")
    dx = ops.gemm_dense(f, w_dec, b_mn=True, bias=b_dec, target=x, res_coef=2.0 / B, out2=recon, loss=loss,
                        colsum=bsum)
    ref = f.float() @ w_dec.float() + b_dec
    _close(recon, ref)
    rf = recon.float()
    ref_loss = ((rf - x.float()) ** 2).sum()
    assert abs(loss.item() - ref_loss.item()) <= 1e-4 * ref_loss.item()
    _close(dx, 2.0 / B * (rf - x.float()))
    # the bias gradient sums the fp32 residual gradient (before dx is rounded to bf16)
    torch.testing.assert_close(bsum, (2.0 / B * (rf - x.float())).sum(0), atol=1e-4, rtol=1e-3)


def test_weight_gradient_with_rank_one_correction_and_sumsq():
    from saelens_b200 import ops

    B, N, D = 1024, 768, 256
    dh = _bf(B, N, scale=0.1, seed=8)                   # [batch, d_sae]: MN-major A for dH^T
    x = _bf(B, D, seed=9)                               # [batch, d_in]: MN-major B
    gb = torch.randn(N, device="cuda")
    b_dec = torch.randn(D, device="cuda")
    sq = torch.zeros(1, device="cuda")
    g = ops.gemm_dense(dh, x, a_mn=True, b_mn=True, r1_row=gb, r1_col=b_dec, sumsq=sq)
    ref = dh.float().T @ x.float() - gb[:, None] * b_dec[None]
    _close(g, ref)
    torch.testing.assert_close(sq, g.float().pow(2).sum().reshape(1), rtol=1e-3, atol=1e-3)


def test_jumprelu_backward_window_gradient():
    from saelens_b200 import ops

    B, D, N = 256, 512, 1024
    dxh = _bf(B, D, scale=0.01, seed=10)
    w_dec = _bf(N, D, scale=0.05, seed=11)
    thr = torch.rand(N, device="cuda") * 0.2 + 0.05
    pre = (thr[None] + torch.randn(B, N, device="cuda") * 0.05).to(torch.bfloat16)  # many entries in the window
    bw, l0c = 0.05, 1.0 / (B * 0.05)
    gthr = torch.zeros(N, device="cuda")
    gb = torch.zeros(N, device="cuda")
    dh = ops.gemm_dense(dxh, w_dec, hin=pre, thr=thr, bandwidth=bw, l0c=l0c, gthr=gthr, colsum=gb)
    df = dxh.float() @ w_dec.float().T
    p = pre.float()
    ref_dh = torch.where(p > thr, df, torch.zeros_like(df))
    _close(dh, ref_dh)
    x = (p - thr) / bw
    win = (x > -0.5) & (x < 0.5)
    ref_g = torch.where(win, -(thr / bw) * df - l0c, torch.zeros_like(df)).sum(0)
    torch.testing.assert_close(gthr, ref_g, atol=2e-2 * ref_g.abs().max().item(), rtol=2e-2)
    torch.testing.assert_close(gb, dh.float().sum(0), atol=1e-3, rtol=1e-2)


def test_gated_dual_path_epilogue():
    from saelens_b200 import ops

    B, D, N = 256, 512, 1024
    x, w = _bf(B, D, seed=12), _bf(N, D, scale=0.05, seed=13)
    b_gate, b_mag = torch.randn(N, device="cuda") * 0.1, torch.randn(N, device="cuda") * 0.1
    r_mag = torch.randn(N, device="cuda") * 0.2
    gate = torch.empty(B, N, dtype=torch.bfloat16, device="cuda")
    f = ops.gemm_dense(x, w, gate_bias=b_gate, mag_scale=r_mag.exp(), bias=b_mag, out2=gate)
    acc = x.float() @ w.float().T
    pg = acc + b_gate
    pm = acc * r_mag.exp() + b_mag
    _close(gate, torch.relu(pg))
    _close(f, torch.where(pg > 0, torch.relu(pm), torch.zeros_like(pm)))


@pytest.mark.parametrize("M, N, K", [(256, 512, 256), (300, 1000, 200), (1024, 2056, 512)])
def test_staged_row_stores_equal_per_thread_stores(monkeypatch, M, N, K):
    """The epilogue's warp-staged row stores (full 32-column chunks through a shared-memory tile)
    write exactly what per-thread stores write, for `out` and `out2`, ragged rows and columns
    included, and nothing past column N."""
    from saelens_b200 import ops

    a, b = _bf(M, K, seed=11), _bf(N, K, seed=12)
    bias = torch.randn(N, device="cuda")
    thr = torch.rand(N, device="cuda") * 0.5
    res = {}
    for staged in ("1", "0"):
        monkeypatch.setenv("SAELENS_B200_GEMM_STAGED_STORE", staged)
        n8 = (N + 7) // 8 * 8 + 8
        buf = torch.full((M, n8), 7.0, dtype=torch.bfloat16, device="cuda")
        buf2 = torch.full((M, n8), 7.0, dtype=torch.bfloat16, device="cuda")
        ops.gemm_dense(a, b, out=buf[:, :N], out2=buf2[:, :N], bias=bias, thr=thr)
        torch.cuda.synchronize()
        assert (buf[:, N:] == 7.0).all() and (buf2[:, N:] == 7.0).all(), "columns past N were written"
        res[staged] = (buf, buf2)
    assert torch.equal(res["1"][0], res["0"][0]) and torch.equal(res["1"][1], res["0"][1])
