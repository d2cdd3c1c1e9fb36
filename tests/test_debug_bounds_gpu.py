"""Debug bounds checks and canary-padded outputs.

The debug module `_C_debug` is the sparse / top-k / ring / router kernel sources compiled with
`-DSB_DEBUG_BOUNDS=1`: every data-dependent index is tested before it is dereferenced, and an
out-of-range one is skipped and recorded (source line, value, bound, count) instead of touching
memory.  Every output in these tests is a view of a larger allocation whose tail rows hold a
canary value, checked after the launch.  Every out-of-range index the tests inject points into
such padding, so even a check that did not fire would read or write padding (and trip a canary
or a value comparison), never memory outside an allocation.
"""

import pytest
import torch

pytestmark = pytest.mark.gpu

CANARY = -77.0  # exact in bf16, fp32 and the integer types
PAD = 8


def _main():
    from saelens_b200.ops._build import load

    return load()


def _dbg():
    from saelens_b200.ops._build import load_debug

    m = load_debug()
    for unit in ("sparse", "topk", "p2p"):
        getattr(m, f"{unit}_bounds_info")(True)  # clear earlier records
    return m


def _padded(shape, dtype, fill=CANARY):
    """(full, view): `view` is the first shape[0] rows of a buffer with PAD canary rows after it."""
    full = torch.full((shape[0] + PAD, *shape[1:]), fill, dtype=dtype, device="cuda")
    return full, full[: shape[0]]


def _canary_intact(full, rows):
    return bool((full[rows:] == CANARY).all())


def _selection(M, N, k, seed=0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    vals = torch.randn(M, k, device="cuda", generator=g)
    idx = torch.stack([torch.randperm(N, device="cuda", generator=g)[:k] for _ in range(M)]).int()
    return vals, idx


def _dense_decode(vals, idx, W, bias):
    M, N = vals.shape[0], W.shape[0]
    live = idx >= 0
    F = torch.zeros(M, N, device="cuda")
    F.scatter_(1, idx.clamp(min=0).long(), torch.where(live, vals.relu(), torch.zeros_like(vals)))
    return F @ W.float() + bias


def _decode(nat, vals, idx, W, bias, x):
    M, D = x.shape
    bufs = {n: _padded((M, D), torch.bfloat16) for n in ("out", "resid", "dxhat")}
    loss_full, loss = _padded((M,), torch.float32)
    bsum_full, bsum = _padded((D,), torch.float32)
    bsum.zero_()
    nat.decode_mse(vals, idx, True, None, W, bias, x, bufs["out"][1], bufs["resid"][1], bufs["dxhat"][1], None,
                   2.0 / M, loss, bsum)
    torch.cuda.synchronize()
    for name, (full, _) in bufs.items():
        assert _canary_intact(full, M), f"{name} canary overwritten"
    assert _canary_intact(loss_full, M) and _canary_intact(bsum_full, D)
    return bufs["out"][1], loss


@pytest.mark.parametrize("which", ["main", "debug"])
def test_decode_canary_padded_outputs(which):
    nat = _main() if which == "main" else _dbg()
    M, N, D, k = 48, 1024, 256, 16
    torch.manual_seed(0)
    W = (torch.randn(N, D, device="cuda") * 0.05).to(torch.bfloat16)
    vals, idx = _selection(M, N, k)
    idx[0, 3] = -1
    bias = torch.randn(D, device="cuda") * 0.1
    x = torch.randn(M, D, device="cuda").to(torch.bfloat16)
    out, loss = _decode(nat, vals, idx, W, bias, x)
    ref = _dense_decode(vals, idx, W, bias)
    assert torch.allclose(out.float(), ref, atol=2e-2, rtol=2e-2)
    assert torch.allclose(loss, (ref - x.float()).pow(2).sum(-1), rtol=2e-2, atol=1e-2)
    if which == "debug":
        assert nat.sparse_bounds_info(True)[3] == 0


def test_debug_decode_skips_and_records_latent_ids_past_the_dictionary():
    dbg = _dbg()
    M, N, D, k = 32, 512, 256, 8
    torch.manual_seed(1)
    w_full = torch.full((N + PAD, D), 100.0, dtype=torch.bfloat16, device="cuda")  # loud if read
    w_full[:N] = (torch.randn(N, D, device="cuda") * 0.05).to(torch.bfloat16)
    W = w_full[:N]
    vals, idx = _selection(M, N, k, seed=1)
    vals = vals.abs() + 0.1  # every entry live
    bad = idx.clone()
    bad[3, 2] = N + 5
    bad[10, 0] = N + PAD - 1
    bias = torch.zeros(D, device="cuda")
    x = torch.randn(M, D, device="cuda").to(torch.bfloat16)
    out, _ = _decode(dbg, vals, bad, W, bias, x)
    line, value, bound, count = dbg.sparse_bounds_info(True)
    assert count == 2 and bound == N and value in (N + 5, N + PAD - 1) and line > 0
    dropped = bad.clone()
    dropped[dropped >= N] = -1
    assert torch.allclose(out.float(), _dense_decode(vals, dropped, W, bias), atol=2e-2, rtol=2e-2)


def _csc(nat, vals, idx, N):
    counts_full, counts = _padded((N,), torch.int32)
    fire_full, fire = _padded((N,), torch.int32)
    counts.zero_()
    fire.zero_()
    nat.csc_count(vals, idx, None, None, counts, fire)
    colptr = torch.zeros(N + 1, dtype=torch.int64, device="cuda")
    torch.cumsum(counts, 0, out=colptr[1:])
    P = vals.numel()
    pairs_full, pairs = _padded((P,), torch.int64)
    cursor = torch.zeros(N, dtype=torch.int32, device="cuda")
    nat.csc_fill(vals, idx, None, None, colptr, cursor, pairs)
    torch.cuda.synchronize()
    assert _canary_intact(counts_full, N) and _canary_intact(fire_full, N) and _canary_intact(pairs_full, P)
    n = int(colptr[-1])
    lists = [sorted(pairs[colptr[j] : colptr[j + 1]].tolist()) for j in range(N)]
    return counts.clone(), colptr, pairs, n, lists


def test_debug_csc_build_drops_out_of_range_ids():
    dbg, main = _dbg(), _main()
    M, N, k = 64, 256, 8
    vals, idx = _selection(M, N, k, seed=2)
    bad = idx.clone()
    bad[5, 1] = N + 2
    bad[40, 7] = N + PAD - 1
    vals[5, 1] = 1.0  # live, so only the id check can drop it
    vals[40, 7] = 1.0
    c_dbg, _, _, n_dbg, l_dbg = _csc(dbg, vals, bad, N)
    line, value, bound, count = dbg.sparse_bounds_info(True)
    assert count == 4 and bound == N and line > 0  # two ids, checked by the count and the fill pass
    dropped = bad.clone()
    dropped[dropped >= N] = -1
    c_ref, _, _, n_ref, l_ref = _csc(main, vals, dropped, N)
    assert torch.equal(c_dbg, c_ref) and n_dbg == n_ref and l_dbg == l_ref


def test_debug_latent_grad_drops_a_corrupt_pair_id():
    dbg, main = _dbg(), _main()
    M, N, D, k = 64, 256, 128, 8
    torch.manual_seed(3)
    # vals / idx are views of padded buffers: pair ids up to (M + PAD) * k - 1 stay inside them
    vals_full = torch.zeros(M + PAD, k, device="cuda")
    idx_full = torch.zeros(M + PAD, k, dtype=torch.int32, device="cuda")
    v, i = _selection(M, N, k, seed=3)
    vals_full[:M], idx_full[:M] = v.abs() + 0.05, i
    vals, idx = vals_full[:M], idx_full[:M]
    _, colptr, pairs, P, lists = _csc(main, vals, idx, N)
    W_dec = (torch.randn(N, D, device="cuda") * 0.05).to(torch.bfloat16)
    W_enc = (torch.randn(N, D, device="cuda") * 0.05).to(torch.bfloat16)
    dxhat = (torch.randn(M, D, device="cuda") * 0.01).to(torch.bfloat16)
    x = torch.randn(M, D, device="cuda").to(torch.bfloat16)

    def run(nat, pr):
        gd_full, gd = _padded((N, D), torch.bfloat16)
        ge_full, ge = _padded((N, D), torch.bfloat16)
        gb_full, gb = _padded((N,), torch.float32)
        nat.latent_grad(colptr, pr, vals, None, None, dxhat, None, x, None, W_dec, W_enc, gd, ge, gb, None, None,
                        None, None, None, idx, None)
        torch.cuda.synchronize()
        assert _canary_intact(gd_full, N) and _canary_intact(ge_full, N) and _canary_intact(gb_full, N)
        return gd.clone(), ge.clone(), gb.clone()

    ref = run(main, pairs)
    js = int(max(range(N), key=lambda j: len(lists[j])))  # a latent with several pairs
    pos = int(colptr[js])
    p_drop = int(pairs[pos])
    corrupt = pairs.clone()
    corrupt[pos] = M * k + 3  # past the pair ids, inside the padded vals / idx buffers
    got = run(dbg, corrupt)
    line, value, bound, count = dbg.sparse_bounds_info(True)
    assert count == 1 and value == M * k + 3 and bound == M * k and line > 0
    others = torch.ones(N, dtype=torch.bool, device="cuda")
    others[js] = False
    for a, b in zip(got, ref):
        assert torch.equal(a[others], b[others])
    # latent js: the reference minus the dropped pair's contribution
    b_row = p_drop // k
    coef = float(vals.flatten()[p_drop])
    dz = float((dxhat[b_row].float() * W_dec[js].float()).sum())
    want_gd = ref[0][js].float() - coef * dxhat[b_row].float()
    want_ge = ref[1][js].float() - dz * x[b_row].float()
    assert torch.allclose(got[0][js].float(), want_gd, atol=2e-3, rtol=2e-2)
    assert torch.allclose(got[1][js].float(), want_ge, atol=2e-2, rtol=2e-2)
    assert abs(float(got[2][js]) - (float(ref[2][js]) - dz)) <= 1e-3 + 1e-3 * abs(float(ref[2][js]))


def test_debug_ring_gather_skips_permutation_rows_past_the_chunk():
    dbg = _dbg()
    R, D = 64, 128
    data = torch.randn(2, R, D, device="cuda").to(torch.bfloat16)  # slot 1 is the padding of slot 0
    slot = torch.zeros(1, dtype=torch.int32, device="cuda")
    perm = torch.randperm(R, device="cuda").int()
    perm[5] = R + 3
    out_full, out = _padded((R, D), torch.bfloat16)
    dbg.ring_gather(data, slot, perm, out)
    torch.cuda.synchronize()
    line, value, bound, count = dbg.p2p_bounds_info(True)
    assert count == 1 and value == R + 3 and bound == R and line > 0
    assert _canary_intact(out_full, R)
    keep = torch.arange(R, device="cuda") != 5
    assert torch.equal(out[keep], data[0][perm[keep].long()])
    assert bool((out[5] == CANARY).all())  # the skipped row was not written


def test_engine_steps_identical_under_debug_bounds(monkeypatch):
    """Fused TopK steps through the bounds-checked kernels: no violations, the same first loss as
    the normal build (the checks change no arithmetic) and the same later losses up to the order
    of the float atomics in the gradient sums."""
    from saelens_b200 import ops
    from saelens_b200.models.topk import TopKTrainingSAE, TopKTrainingSAEConfig
    from saelens_b200.training.engine import FusedTopKEngine

    def losses(debug: bool) -> list[float]:
        if debug:
            monkeypatch.setenv("SAELENS_B200_DEBUG_BOUNDS", "1")
        else:
            monkeypatch.delenv("SAELENS_B200_DEBUG_BOUNDS", raising=False)
        torch.manual_seed(0)
        sae = TopKTrainingSAE(TopKTrainingSAEConfig(d_in=256, d_sae=4096, k=32, device="cuda"))
        eng = FusedTopKEngine(sae, lr=1e-3)
        assert bool(getattr(eng.native, "debug_bounds", False)) == debug
        x = torch.randn(512, 256, device="cuda").to(torch.bfloat16)
        out = [float(eng.step(x).loss) for _ in range(3)]
        eng.status.check()
        return out

    _dbg()
    ref = losses(False)
    got = losses(True)
    assert ops.bounds_violations() == {}
    assert got[0] == ref[0]
    assert all(abs(a - b) <= 1e-4 * abs(b) for a, b in zip(got, ref))
