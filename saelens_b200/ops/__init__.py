"""Native sm_100a operators.

`native()` returns the compiled extension; every wrapper here calls it directly, so a missing
build fails loudly on a CUDA machine instead of silently running a PyTorch fallback.  The
PyTorch paths of the models (`saelens_b200.models`) compute the same quantities on any device
and serve as the oracle of the GPU tests.
"""

from __future__ import annotations

import os

import torch

from saelens_b200.ops._build import load as _load
from saelens_b200.ops.status import StatusWord

__all__ = [
    "native",
    "available",
    "bounds_violations",
    "debug_bounds_enabled",
    "gemm_tn",
    "row_topk",
    "decode_mse",
    "attention",
    "gather_rows",
    "StatusWord",
]


class _DebugBoundsNative:
    """The extension with its index-dereferencing kernels taken from the debug-bounds module
    (`_C_debug`: every data-dependent index checked before use, violations skipped and recorded;
    read them with `bounds_violations()`), everything else from the main module."""

    def __init__(self) -> None:
        from saelens_b200.ops._build import load_debug

        self._main = _load()
        self._debug = load_debug()

    def __getattr__(self, name: str):
        return getattr(self._debug, name) if hasattr(self._debug, name) else getattr(self._main, name)


_DEBUG_NATIVE: _DebugBoundsNative | None = None


def debug_bounds_enabled() -> bool:
    return os.environ.get("SAELENS_B200_DEBUG_BOUNDS", "0") not in ("", "0")


def native():
    """The compiled extension; with SAELENS_B200_DEBUG_BOUNDS=1 its index-dereferencing kernels
    come from the bounds-checked debug module."""
    global _DEBUG_NATIVE
    if debug_bounds_enabled():
        if _DEBUG_NATIVE is None:
            _DEBUG_NATIVE = _DebugBoundsNative()
        return _DEBUG_NATIVE
    return _load()


def bounds_violations(reset: bool = True) -> dict[str, dict[str, int]]:
    """Bounds violations recorded by the debug-bounds module since the last reset, per source
    file: {file: {line, value, bound, count}} of the first violation (empty when none)."""
    from saelens_b200.ops._build import load_debug

    dbg = load_debug()
    out: dict[str, dict[str, int]] = {}
    for unit in ("sparse", "topk", "p2p"):
        line, value, bound, count = getattr(dbg, f"{unit}_bounds_info")(reset)
        if count:
            out[f"{unit}.cu"] = {"line": line, "value": value, "bound": bound, "count": count}
    return out


def available() -> bool:
    """True when the extension is built and a CUDA device is present."""
    if not torch.cuda.is_available():
        return False
    try:
        _load()
    except ImportError:
        return False
    return True


def gemm_tn(
    a: torch.Tensor,
    b: torch.Tensor,
    bias: torch.Tensor | None = None,
    scale: torch.Tensor | None = None,
    relu: bool = False,
    out: torch.Tensor | None = None,
    chunk_max: bool = False,
    status: StatusWord | None = None,
    max_ctas: int = 0,
) -> tuple[torch.Tensor | None, torch.Tensor | None]:
    """`epilogue(a @ b.T)` on the tcgen05 tensor cores.

    a: [M, K] bf16, b: [N, K] bf16 (K contiguous, K % 8 == 0; any N, with N % 256 == 0 when
    `chunk_max` is set).  Epilogue: `(acc + bias) * scale`, optional ReLU, rounded to bf16.  With
    `chunk_max` it also returns the max of every 32-column chunk ([M, N/32] bf16).  When N is not
    a multiple of 8 the result is a view of rows padded to a multiple of 8 (16-byte rows).
    """
    M, N = a.shape[0], b.shape[0]
    if out is None:
        n_alloc = (N + 7) // 8 * 8
        out = torch.empty(M, n_alloc, dtype=torch.bfloat16, device=a.device)[:, :N]
    cmax = torch.empty(M, N // 32, dtype=torch.bfloat16, device=a.device) if chunk_max else None
    st = status or StatusWord(a.device)
    native().gemm_tn_bf16(a, b, bias, scale, relu, out, cmax, st.tensor, max_ctas)
    if status is None:
        st.check("gemm_tn")
    return out, cmax


def row_topk(
    h: torch.Tensor,
    cmax: torch.Tensor,
    k: int,
    k_dev: torch.Tensor | None = None,
    mask_words: torch.Tensor | None = None,
    status: StatusWord | None = None,
) -> tuple[torch.Tensor, torch.Tensor]:
    """Exact per-row top-k of bf16 `h` ([M, N]) using its chunk maxima `cmax` ([M, N/32]).

    Returns (values fp32 [M, k], indices int32 [M, k]); unused slots hold index -1.
    Ties at the k-th value are broken by the smaller column index.
    """
    M = h.shape[0]
    vals = torch.empty(M, k, dtype=torch.float32, device=h.device)
    idx = torch.empty(M, k, dtype=torch.int32, device=h.device)
    st = status or StatusWord(h.device)
    native().row_topk(h, cmax, k, k_dev, mask_words, vals, idx, st.tensor)
    if status is None:
        st.check("row_topk")
    return vals, idx


def decode_mse(
    vals: torch.Tensor,
    idx: torch.Tensor,
    w: torch.Tensor,
    target: torch.Tensor,
    inv_scale: torch.Tensor | None = None,
    bias: torch.Tensor | None = None,
    relu: bool = True,
    want_out: bool = True,
    want_resid: bool = False,
    grad_coef: float = 0.0,
    grad_coef_dev: torch.Tensor | None = None,
    want_bsum: bool = False,
) -> dict[str, torch.Tensor]:
    """Sparse decode `sum_i a_i w[idx_i] + bias` and its squared error against `target`."""
    M, D = target.shape
    dev = target.device
    res: dict[str, torch.Tensor] = {}
    out = torch.empty(M, D, dtype=torch.bfloat16, device=dev) if want_out else None
    resid = torch.empty(M, D, dtype=torch.bfloat16, device=dev) if want_resid else None
    dx = torch.empty(M, D, dtype=torch.bfloat16, device=dev) if (grad_coef != 0.0) else None
    loss_row = torch.empty(M, dtype=torch.float32, device=dev)
    bsum = torch.zeros(D, dtype=torch.float32, device=dev) if want_bsum else None
    native().decode_mse(
        vals, idx, relu, inv_scale, w, bias, target, out, resid, dx, grad_coef_dev,
        float(grad_coef), loss_row, bsum,
    )
    res["loss_row"] = loss_row
    if out is not None:
        res["out"] = out
    if resid is not None:
        res["resid"] = resid
    if dx is not None:
        res["dxhat"] = dx
    if bsum is not None:
        res["bsum"] = bsum
    return res


def attention(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    scale: float,
    softcap: float | None = None,
    causal: bool = True,
    out: torch.Tensor | None = None,
    status: StatusWord | None = None,
) -> torch.Tensor:
    """Prefill attention on the tcgen05 tensor cores.

    q: [B, S, H, D], k / v: [B, S, KV, D] bf16 (head dim contiguous, heads adjacent within a
    token; H a multiple of KV, query head h reads K/V head h // (H / KV)).  Returns
    softmax(cap(q k^T * scale)) v as [B, S, H, D] bf16, causal unless `causal=False`, with
    cap(x) = softcap * tanh(x / softcap) when `softcap` is given.  D in {64, 128, 256}.
    """
    if q.dim() != 4 or q.shape[-1] not in (64, 128, 256):
        raise ValueError(f"attention: head dim must be 64, 128 or 256, got shape {tuple(q.shape)}")
    if k.shape[2] < 1 or q.shape[2] % k.shape[2]:
        raise ValueError("attention: query heads must be a multiple of the K/V heads")
    if out is None:
        out = torch.empty(q.shape, dtype=torch.bfloat16, device=q.device)
    st = status or StatusWord(q.device)
    native().attention_fwd(q, k, v, out, float(scale), float(softcap or 0.0), bool(causal), st.tensor)
    if status is None:
        st.check("attention")
    return out


def gemm_dense(
    a: torch.Tensor,
    b: torch.Tensor,
    a_mn: bool = False,
    b_mn: bool = False,
    out: torch.Tensor | None = None,
    want_out: bool = True,
    status: StatusWord | None = None,
    **epi: object,
) -> torch.Tensor | None:
    """Dense GEMM of the dense SAE steps on tcgen05: `epilogue(A @ B^T)` with A given as [M, K]
    (or [K, M] when `a_mn`) and B as [N, K] (or [K, N] when `b_mn`), bf16.

    Epilogue keywords (all optional, see `gemm_dense_bf16`): out2, bias, r1_row / r1_col, thr,
    relu, hin / bandwidth / l0c / gthr (JumpReLU backward), target / res_coef / loss (residual),
    colsum, colcnt, nnz, sumsq, gate_bias / mag_scale (gated SAE), rs_bases / rs_rank / rs_off / rs_n
    (reduce-scatter: rows stored into their owners' landing slots over NVLink, with
    `want_out=False`).  Returns `out` ([M, N] bf16), or None with `want_out=False`.
    """
    M = a.shape[1] if a_mn else a.shape[0]
    N = b.shape[1] if b_mn else b.shape[0]
    if out is None and want_out:
        n_alloc = (N + 7) // 8 * 8
        out = torch.empty(M, n_alloc, dtype=torch.bfloat16, device=a.device)[:, :N]
    st = status or StatusWord(a.device)
    native().gemm_dense_bf16(a, a_mn, b, b_mn, out=out if want_out else None, status=st.tensor, **epi)
    if status is None:
        st.check("gemm_dense")
    return out


def gather_rows(a: torch.Tensor, b: torch.Tensor | None = None, perm: torch.Tensor | None = None,
                out: torch.Tensor | None = None) -> torch.Tensor:
    """`torch.cat([a, b])[perm]` in one pass on the device (rows moved as raw bytes, warp per
    row).  `perm` is int64 on the device; without it the first `len(out)` rows are copied.
    Indices outside the two sources leave their output row untouched."""
    n = (a.shape[0] + (0 if b is None else b.shape[0])) if perm is None else perm.shape[0]
    if out is None:
        out = torch.empty((n, *a.shape[1:]), dtype=a.dtype, device=a.device)
    native().gather_rows(a, b, perm, out)
    return out
