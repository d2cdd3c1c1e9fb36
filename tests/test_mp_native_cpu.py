"""CPU checks of the arithmetic the native matching-pursuit kernels implement (ops/csrc/mp.cu).

The kernels replace the reference loop (sae_lens/saes/matching_pursuit_sae.py:258-335) by
  * a per-row step: value = relu(<r, W[i]>), codes[i] += value, r -= value * W[i], and the row
    stops when no new latent was added (instead of comparing whole support masks) or when |r| is
    below the threshold;
  * a reverse replay for the gradient: g_v = g[i] - <G, W[i]>, dW[i] += g_v r_t - v G,
    G += g_v W[i], with r_t rebuilt as r_{t+1} + v W[i].
Both are restated here in float64 and compared with the reference loop and its autograd.
"""

from __future__ import annotations

import pytest
import torch

from saelens_b200.models.matching_pursuit import _encode_matching_pursuit_torch


def _kernel_forward(x: torch.Tensor, W: torch.Tensor, thresh: float, iters: int, stop_dup: bool):
    """The step kernel's semantics, one row at a time, recording picks and values."""
    B, _ = x.shape
    N = W.shape[0]
    r = x.clone()
    acts = torch.zeros(B, N, dtype=x.dtype)
    done = torch.zeros(B, dtype=torch.bool)
    idx, val = [], []
    for _ in range(iters):
        it_i = torch.full((B,), -1, dtype=torch.int64)
        it_v = torch.zeros(B, dtype=x.dtype)
        for b in range(B):
            if done[b]:
                continue
            i = int((r[b] @ W.T).relu().argmax())
            v = float((r[b] * W[i]).sum().relu())
            old = float(acts[b, i])
            acts[b, i] = old + v
            r[b] = r[b] - v * W[i]
            added = old == 0.0 and old + v != 0.0
            if (stop_dup and not added) or (thresh > 0 and float(r[b].norm()) < thresh):
                done[b] = True
            it_i[b], it_v[b] = i, v
        idx.append(it_i)
        val.append(it_v)
        if bool(done.all()):
            break
    return acts, r, torch.stack(idx), torch.stack(val)


def _kernel_backward(r_final: torch.Tensor, g_acts: torch.Tensor, idx: torch.Tensor, val: torch.Tensor,
                     W: torch.Tensor):
    r = r_final.clone()
    G = torch.zeros_like(r)
    gW = torch.zeros_like(W)
    for t in range(idx.shape[0] - 1, -1, -1):
        for b in range(r.shape[0]):
            v, i = float(val[t, b]), int(idx[t, b])
            if not v > 0 or i < 0:
                continue
            w = W[i]
            gv = g_acts[b, i] - (G[b] * w).sum()
            r_t = r[b] + v * w
            gW[i] += gv * r_t - v * G[b]
            G[b] = G[b] + gv * w
            r[b] = r_t
    return G, gW


def _problem(seed: int, B: int = 6, D: int = 16, N: int = 40):
    g = torch.Generator().manual_seed(seed)
    W = torch.randn(N, D, generator=g, dtype=torch.float64)
    W = W / W.norm(dim=1, keepdim=True)
    x = torch.randn(B, D, generator=g, dtype=torch.float64)
    return x, W


@pytest.mark.parametrize("stop_dup,thresh,iters", [(True, 0.0, 16), (False, 0.5, 12), (True, 0.3, 16),
                                                   (False, 0.0, 5)])
def test_step_semantics_match_reference_loop(stop_dup: bool, thresh: float, iters: int) -> None:
    x, W = _problem(0)
    want = _encode_matching_pursuit_torch(x, W, thresh, iters, stop_dup)
    got, _, _, _ = _kernel_forward(x, W, thresh, iters, stop_dup)
    torch.testing.assert_close(got, want, rtol=1e-12, atol=1e-12)


@pytest.mark.parametrize("stop_dup,thresh,iters", [(True, 0.0, 16), (False, 0.4, 10), (False, 0.0, 6)])
def test_replayed_backward_matches_autograd(stop_dup: bool, thresh: float, iters: int) -> None:
    x, W = _problem(1)
    acts, r_final, idx, val = _kernel_forward(x, W, thresh, iters, stop_dup)
    g_acts = torch.randn(acts.shape, dtype=torch.float64, generator=torch.Generator().manual_seed(7))
    g_acts = g_acts * (torch.rand(acts.shape, generator=torch.Generator().manual_seed(8)) < 0.5)

    xr = x.clone().requires_grad_(True)
    Wr = W.clone().requires_grad_(True)
    picks = [idx[t] for t in range(idx.shape[0])]
    out = _encode_matching_pursuit_torch(xr, Wr, thresh, iters, stop_dup, picks=picks)
    torch.testing.assert_close(out.detach(), acts, rtol=1e-12, atol=1e-12)
    (out * g_acts).sum().backward()

    g_in, g_W = _kernel_backward(r_final, g_acts, idx, val, W)
    torch.testing.assert_close(g_in, xr.grad, rtol=1e-9, atol=1e-9)
    torch.testing.assert_close(g_W, Wr.grad, rtol=1e-9, atol=1e-9)


def test_native_dispatch_stays_off_on_cpu() -> None:
    from saelens_b200.ops import mp

    x, W = _problem(2)
    assert not mp.native_supported(x.float(), W.float())
