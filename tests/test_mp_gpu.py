"""Native matching-pursuit encode on the GPU (ops/mp.py, ops/csrc/mp.cu, the score GEMM's argmax
epilogue in ops/csrc/gemm_tc.cu) against the PyTorch loop of the reference's iteration
(sae_lens/saes/matching_pursuit_sae.py:258-335) run in fp32 with the same picks."""

from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():
    pytest.skip("needs a CUDA device", allow_module_level=True)

from saelens_b200 import ops  # noqa: E402
from saelens_b200.models.matching_pursuit import _encode_matching_pursuit_torch  # noqa: E402
from saelens_b200.ops import mp  # noqa: E402


def _decode_keys(key: torch.Tensor) -> torch.Tensor:
    return 0xFFFFFFFF - (key & 0xFFFFFFFF)


@pytest.mark.parametrize("M,N,K", [(300, 4099, 256), (1000, 8192, 512), (2048, 3000, 128)])
def test_gemm_row_argmax_epilogue(M: int, N: int, K: int) -> None:
    g = torch.Generator(device="cuda").manual_seed(M + N)
    a = torch.randn(M, K, device="cuda", generator=g).bfloat16()
    b = torch.randn(N, K, device="cuda", generator=g).bfloat16()
    a[7] = -a[7].abs()
    b_neg = b.clone()
    key = torch.zeros(M, dtype=torch.int64, device="cuda")
    st = ops.StatusWord("cuda")
    ops.native().gemm_tn_bf16(a, b_neg, None, None, True, None, None, st.tensor, 0, None, key)
    st.check("argmax gemm")
    idx = _decode_keys(key)
    assert bool((key != 0).all())
    scores = (a.float() @ b.float().T).relu()
    best = scores.max(dim=1).values
    picked = scores.gather(1, idx.unsqueeze(1)).squeeze(1)
    # fp32 accumulation in another order: the pick is a maximum up to rounding
    assert bool((picked >= best - 1e-3 * best.abs().clamp_min(1.0)).all())
    agree = (idx == scores.argmax(dim=1)).float().mean().item()
    assert agree > 0.99
    zero_rows = best == 0
    if bool(zero_rows.any()):  # every score <= 0: the first column, as torch's argmax of zeros
        assert bool((idx[zero_rows] == 0).all())


def _dictionary(N: int, D: int, seed: int, dtype=torch.float32):
    g = torch.Generator(device="cuda").manual_seed(seed)
    W = torch.randn(N, D, device="cuda", generator=g)
    W = W / W.norm(dim=1, keepdim=True)
    codes = torch.zeros(512, N, device="cuda")
    cols = torch.randint(0, N, (512, 6), device="cuda", generator=g)
    codes.scatter_(1, cols, torch.rand(512, 6, device="cuda", generator=g) * 3 + 0.5)
    x = codes @ W + 0.01 * torch.randn(512, D, device="cuda", generator=g)
    return x, W.to(dtype)


@pytest.mark.parametrize("stop_dup,thresh,iters", [(True, 0.0, None), (False, 0.05, 40), (True, 0.05, None),
                                                   (False, 0.0, 12)])
def test_native_forward_matches_reference_loop_with_same_picks(stop_dup, thresh, iters) -> None:
    x, W = _dictionary(2048, 256, 0)
    acts, resid, idx, val = mp.trace_matching_pursuit(x, W, thresh, iters, stop_dup)
    picks = [idx[t] for t in range(idx.shape[0])]
    want = _encode_matching_pursuit_torch(x, W, thresh, iters, stop_dup, picks=picks)
    torch.testing.assert_close(acts, want, rtol=1e-4, atol=1e-4)
    torch.testing.assert_close(resid, x - acts @ W, rtol=1e-3, atol=1e-3)
    # the run stops where the reference stops: rows that were still running at the end agree
    plain = _encode_matching_pursuit_torch(x, W, thresh, iters, stop_dup)
    rel = ((x - acts @ W).norm(dim=1) / x.norm(dim=1)).mean()
    rel_ref = ((x - plain @ W).norm(dim=1) / x.norm(dim=1)).mean()
    assert float(rel) <= float(rel_ref) * 1.05 + 1e-4


def test_native_encode_recovers_sparse_codes() -> None:
    # six atoms per row plus noise: most rows stop after the six (the median L0 is 6); a row whose
    # noise keeps finding new atoms runs on, as the reference loop's does
    x, W = _dictionary(4096, 512, 1)
    acts = mp.encode_matching_pursuit(x, W, 0.05, None, True)
    l0 = (acts != 0).sum(dim=1).float()
    l0_ref = (_encode_matching_pursuit_torch(x, W, 0.05, None, True) != 0).sum(dim=1).float()
    assert float(l0.median()) == 6.0
    assert abs(float(l0.mean()) - float(l0_ref.mean())) <= 0.1 * float(l0_ref.mean()) + 0.5
    rel = ((x - acts @ W).norm(dim=1) / x.norm(dim=1)).mean()
    assert float(rel) < 0.1


@pytest.mark.parametrize("wdtype", [torch.float32, torch.bfloat16])
def test_native_backward_matches_autograd_with_same_picks(wdtype) -> None:
    x, W = _dictionary(1024, 128, 2, dtype=wdtype)
    _, _, idx, _ = mp.trace_matching_pursuit(x, W, 0.05, 24, True)
    picks = [idx[t] for t in range(idx.shape[0])]
    g_out = torch.randn(x.shape[0], W.shape[0], device="cuda") * (torch.rand(x.shape[0], W.shape[0],
                                                                             device="cuda") < 0.3)

    xn = x.clone().requires_grad_(True)
    Wn = W.clone().requires_grad_(True)
    acts = mp.encode_matching_pursuit(xn, Wn, 0.05, 24, True)
    (acts.float() * g_out).sum().backward()

    xr = x.clone().requires_grad_(True)
    Wr = W.float().clone().requires_grad_(True)
    ref = _encode_matching_pursuit_torch(xr, Wr, 0.05, 24, True, picks=picks)
    (ref * g_out).sum().backward()

    torch.testing.assert_close(acts.float(), ref.detach(), rtol=1e-3, atol=1e-3)
    torch.testing.assert_close(xn.grad, xr.grad, rtol=2e-3, atol=2e-3)
    torch.testing.assert_close(Wn.grad.float(), Wr.grad, rtol=2e-2 if wdtype == torch.bfloat16 else 2e-3,
                               atol=2e-2 if wdtype == torch.bfloat16 else 2e-3)


def test_training_sae_runs_the_native_encode() -> None:
    from saelens_b200.models.matching_pursuit import MatchingPursuitTrainingSAE, MatchingPursuitTrainingSAEConfig
    from saelens_b200.models.sae import TrainStepInput

    cfg = MatchingPursuitTrainingSAEConfig(d_in=256, d_sae=2048, device="cuda", residual_threshold=0.05)
    sae = MatchingPursuitTrainingSAE(cfg)
    x, _ = _dictionary(2048, 256, 3)
    out = sae.training_forward_pass(TrainStepInput(sae_in=x, coefficients={}, dead_neuron_mask=None,
                                                   n_training_steps=0, is_logging_step=True))
    out.loss.backward()
    assert sae.W_dec.grad is not None and bool(torch.isfinite(sae.W_dec.grad).all())
    assert float(out.metrics["residual_norm"]) < float(x.norm(dim=1).mean())


def test_row_compaction_changes_nothing(monkeypatch) -> None:
    x, W = _dictionary(4096, 256, 4)
    x = torch.cat([x] * 8)  # 4096 rows: compaction triggers once fewer than half still run
    x = x + 0.01 * torch.randn_like(x)
    monkeypatch.setenv("SAELENS_B200_MP_COMPACT", "0")
    a0, r0, i0, v0 = mp.trace_matching_pursuit(x, W, 0.05, 64, True)
    monkeypatch.setenv("SAELENS_B200_MP_COMPACT", "1")
    a1, r1, i1, v1 = mp.trace_matching_pursuit(x, W, 0.05, 64, True)
    assert i0.shape == i1.shape
    assert torch.equal(i0, i1) and torch.equal(v0, v1)
    assert torch.equal(a0, a1) and torch.equal(r0, r1)
