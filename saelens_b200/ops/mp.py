"""Native matching-pursuit encode (sae_lens/saes/matching_pursuit_sae.py:258-335).

Each iteration runs two kernels: the tcgen05 score GEMM `relu(bf16(residual) @ bf16(W_dec)^T)`
with the row argmax fused into its epilogue (the [rows, d_sae] score matrix is never stored), and
`mp_step`, which adds `relu(<residual, W_dec[i]>)` (fp32) to the codes, updates the residual and
stops rows the way the reference does (no new latent added, or residual norm below the threshold).
Stopped rows are skipped by later iterations, as the reference masks them, so running an iteration
after every row has stopped changes nothing; the host therefore reads the running-row count of
iteration t while iteration t + 1 is already queued, and never waits on the device per iteration.

Selection differs from the reference only in precision: the argmax is taken over scores computed
from bf16 operands with fp32 accumulation, and the value added is the exact fp32 inner product of
the residual with the picked decoder row.  With gradients enabled the iterations' picks and values
are recorded and `mp_backward` replays them in reverse (see ops/csrc/mp.cu), giving the gradient
of the codes with respect to the centred input and W_dec that autograd of the reference loop gives
for the same picks.
"""

from __future__ import annotations

import os

import torch

from saelens_b200.ops.status import StatusWord


def native_supported(sae_in_centered: torch.Tensor, W_dec: torch.Tensor) -> bool:
    """True when the native encode applies: CUDA tensors, d_in a multiple of 8 (16-byte bf16 rows
    for the GEMM's tensor maps), fp32 or bf16 decoder, and not disabled by
    SAELENS_B200_MP_NATIVE=0."""
    if os.environ.get("SAELENS_B200_MP_NATIVE", "1") == "0":
        return False
    return (sae_in_centered.is_cuda and W_dec.is_cuda and W_dec.dim() == 2 and W_dec.shape[1] % 8 == 0
            and W_dec.dtype in (torch.float32, torch.bfloat16))


_COMPACT_MIN_ROWS = 256  # no compaction below one CTA-pair tile of rows


def _compaction_enabled() -> bool:
    return os.environ.get("SAELENS_B200_MP_COMPACT", "1") != "0"


def _run(resid0: torch.Tensor, W_dec: torch.Tensor, residual_threshold: float, max_iterations: int,
         stop_on_duplicate_support: bool, record: bool):
    """The forward iterations.  Returns (codes fp32 [B, N], final residual fp32 [B, D], picks
    int32 [T, B] or None, values fp32 [T, B] or None).

    Once at most half of the rows still run (and at least `_COMPACT_MIN_ROWS` would remain), the
    running rows are gathered into smaller residual buffers, so later score GEMMs multiply only
    those; `rows` maps them back to their rows of the codes and of the trace.  Stopped rows are
    skipped by every later iteration anyway, so this changes no result."""
    from saelens_b200.ops import native

    nat = native()
    B, D = resid0.shape
    N = W_dec.shape[0]
    dev = resid0.device
    resid_full = resid0.detach().to(torch.float32).contiguous().clone()
    acts = torch.zeros(B, N, dtype=torch.float32, device=dev)
    if B == 0 or max_iterations <= 0:
        return acts, resid_full, None, None
    W = W_dec.detach().contiguous()
    W_bf = W if W.dtype == torch.bfloat16 else W.to(torch.bfloat16)
    resid = resid_full  # the running rows' residuals (all rows until the first compaction)
    resid_bf = resid.to(torch.bfloat16)
    rows: torch.Tensor | None = None  # int32 original row of each running row (None: identity)
    key = torch.zeros(B, dtype=torch.int64, device=dev)
    done = torch.zeros(B, dtype=torch.uint8, device=dev)
    counts = torch.zeros(max_iterations, dtype=torch.int32, device=dev)
    idx = torch.full((max_iterations, B), -1, dtype=torch.int32, device=dev) if record else None
    val = torch.zeros(max_iterations, B, dtype=torch.float32, device=dev) if record else None
    stops = stop_on_duplicate_support or residual_threshold > 0
    compact = stops and _compaction_enabled()
    host = torch.empty(max_iterations, dtype=torch.int32, pin_memory=True) if stops else None
    events: list[torch.cuda.Event] = []
    st = StatusWord(dev)
    T = 0
    for t in range(max_iterations):
        nat.gemm_tn_bf16(resid_bf, W_bf, None, None, True, None, None, st.tensor, 0, None, key)
        nat.mp_step(resid, resid_bf, key, acts, done, idx[t] if record else None, val[t] if record else None,
                    counts[t:t + 1], W, float(residual_threshold), bool(stop_on_duplicate_support), rows)
        T = t + 1
        if not stops:
            continue
        host[t:t + 1].copy_(counts[t:t + 1], non_blocking=True)
        ev = torch.cuda.Event()
        ev.record()
        events.append(ev)
        if t == 0:
            continue
        events[t - 1].synchronize()
        running = int(host[t - 1])
        if running == 0:
            T = t  # iteration t ran with every row stopped: it added nothing
            break
        M = resid.shape[0]
        if compact and t + 1 < max_iterations and running <= M // 2 and running >= _COMPACT_MIN_ROWS:
            keep = torch.nonzero(done == 0).squeeze(1)  # rows still running after iteration t
            if keep.numel() == 0:
                continue
            if rows is not None:  # the rows that leave keep their final residual in resid_full
                resid_full.index_copy_(0, rows.long(), resid)
            new_rows = keep.to(torch.int32) if rows is None else rows.index_select(0, keep)
            resid = resid.index_select(0, keep)
            resid_bf = resid_bf.index_select(0, keep)
            rows = new_rows.contiguous()
            key = torch.zeros(rows.numel(), dtype=torch.int64, device=dev)
            done = torch.zeros(rows.numel(), dtype=torch.uint8, device=dev)
    if rows is not None:
        resid_full.index_copy_(0, rows.long(), resid)
    st.check("matching pursuit score GEMM")
    if record:
        return acts, resid_full, idx[:T], val[:T]
    return acts, resid_full, None, None


class _MatchingPursuitEncode(torch.autograd.Function):
    @staticmethod
    def forward(ctx, resid0, W_dec, residual_threshold, max_iterations, stop_on_duplicate_support):
        acts, resid, idx, val = _run(resid0, W_dec, residual_threshold, max_iterations,
                                     stop_on_duplicate_support, record=True)
        ctx.save_for_backward(resid, W_dec, idx if idx is not None else torch.empty(0, resid0.shape[0],
                                                                                     dtype=torch.int32,
                                                                                     device=resid0.device),
                              val if val is not None else torch.empty(0, resid0.shape[0], dtype=torch.float32,
                                                                      device=resid0.device))
        ctx.in_dtype = resid0.dtype
        return acts

    @staticmethod
    def backward(ctx, g_acts):
        from saelens_b200.ops import native

        resid, W_dec, idx, val = ctx.saved_tensors
        need_in, need_w = ctx.needs_input_grad[0], ctx.needs_input_grad[1]
        B, D = resid.shape
        r = resid.clone()
        g_resid = torch.zeros(B, D, dtype=torch.float32, device=resid.device)
        g_W = torch.zeros(W_dec.shape, dtype=torch.float32, device=resid.device) if need_w else None
        if idx.shape[0] > 0:
            native().mp_backward(r, g_resid, g_acts.to(torch.float32).contiguous(), idx, val, g_W,
                                 W_dec.detach().contiguous())
        g_in = g_resid.to(ctx.in_dtype) if need_in else None
        g_w_out = g_W.to(W_dec.dtype) if need_w else None
        return g_in, g_w_out, None, None, None


def encode_matching_pursuit(sae_in_centered: torch.Tensor, W_dec: torch.Tensor, residual_threshold: float,
                            max_iterations: int | None, stop_on_duplicate_support: bool) -> torch.Tensor:
    """Dense codes [..., d_sae] of `sae_in_centered` [..., d_in] (same contract as the reference's
    `_encode_matching_pursuit`; the codes have the input's dtype)."""
    shape = sae_in_centered.shape
    x = sae_in_centered.reshape(-1, shape[-1]) if sae_in_centered.ndim != 2 else sae_in_centered
    iters = W_dec.shape[1] if max_iterations is None else int(max_iterations)
    grad = torch.is_grad_enabled() and (x.requires_grad or W_dec.requires_grad)
    if grad:
        acts = _MatchingPursuitEncode.apply(x, W_dec, float(residual_threshold), iters,
                                            bool(stop_on_duplicate_support))
    else:
        acts = _run(x, W_dec, float(residual_threshold), iters, bool(stop_on_duplicate_support), record=False)[0]
    acts = acts.to(sae_in_centered.dtype)
    if sae_in_centered.ndim != 2:
        acts = acts.reshape(*shape[:-1], acts.shape[-1])
    return acts


def trace_matching_pursuit(sae_in_centered: torch.Tensor, W_dec: torch.Tensor, residual_threshold: float,
                           max_iterations: int | None, stop_on_duplicate_support: bool):
    """The native forward with its per-iteration picks and values ([T, B] each), for tests and
    diagnostics: (codes, final residual, picks, values)."""
    iters = W_dec.shape[1] if max_iterations is None else int(max_iterations)
    with torch.no_grad():
        return _run(sae_in_centered, W_dec, float(residual_threshold), iters, bool(stop_on_duplicate_support),
                    record=True)
