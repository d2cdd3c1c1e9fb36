"""The allocation-free CSC entry point (`sb_csc_build_noalloc`, called through its exported C
symbol) against the allocating path the training engine uses (`csc_count`, a prefix sum and
`csc_fill`).  Kept in a file that sorts last so a stop-at-first-failure run has already run
every other test."""

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def _lib():
    from saelens_b200.ops._build import _so_path

    path = _so_path()
    assert path is not None, "native extension not built"
    lib = ctypes.CDLL(path)
    fn = lib.sb_csc_build_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int32, ctypes.c_void_p,
                   ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
    lib.sb_noalloc_strerror.restype = ctypes.c_char_p
    lib.sb_noalloc_strerror.argtypes = [ctypes.c_int]
    return lib, fn


def _random_selection(M, k, N, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    vals = torch.randn(M, k, device="cuda", generator=g)
    idx = torch.argsort(torch.rand(M, N, device="cuda", generator=g), dim=1)[:, :k].to(torch.int32)
    idx[::7, 3] = -1  # empty slots are skipped
    return vals.contiguous(), idx.contiguous()


def _reference(vals, idx, N):
    from saelens_b200 import ops

    nat = ops.native()
    counts = torch.zeros(N, dtype=torch.int32, device="cuda")
    nat.csc_count(vals, idx, None, None, counts, None)
    colptr = torch.zeros(N + 1, dtype=torch.int64, device="cuda")
    torch.cumsum(counts, 0, out=colptr[1:])
    cursor = torch.zeros(N, dtype=torch.int32, device="cuda")
    pairs = torch.full((vals.numel(),), -1, dtype=torch.int64, device="cuda")
    nat.csc_fill(vals, idx, None, None, colptr, cursor, pairs)
    return colptr, pairs


def _canonical(colptr, pairs):
    """Pairs sorted within each latent (the order inside a latent is unspecified)."""
    nnz = int(colptr[-1])
    col = torch.repeat_interleave(torch.arange(colptr.numel() - 1, device="cuda"), colptr[1:] - colptr[:-1])
    key = col * (1 << 40) + pairs[:nnz]
    return torch.sort(key).values


def _call(fn, vals, idx, N, bad=None):
    M = vals.numel()
    colptr = torch.full((N + 1,), -5, dtype=torch.int64, device="cuda")
    pairs = torch.full((max(M, 1),), -5, dtype=torch.int64, device="cuda")
    rc = fn(vals.data_ptr() if M else 0, idx.data_ptr() if M else 0, M, N, colptr.data_ptr(), pairs.data_ptr(),
            bad.data_ptr() if bad is not None else 0, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    return rc, colptr, pairs


@pytest.mark.parametrize("M, k, N", [
    (1024, 32, 8192),      # whole scan blocks
    (512, 16, 1000),       # a partial last scan block
    (256, 64, 1 << 20),    # the maximum: the single-block scan of 1024 block sums is full
])
def test_noalloc_csc_matches_allocating_path_twice(M, k, N):
    lib, fn = _lib()
    bad = torch.full((1,), -7, dtype=torch.int32, device="cuda")
    for call, seed in enumerate((1, 2)):  # two calls in a row: the shared scratch is reused
        vals, idx = _random_selection(M, k, N, seed)
        ref_colptr, ref_pairs = _reference(vals, idx, N)
        rc, colptr, pairs = _call(fn, vals, idx, N, bad)
        assert rc == 0, lib.sb_noalloc_strerror(rc)
        assert torch.equal(colptr, ref_colptr), f"call {call}: colptr differs"
        assert torch.equal(_canonical(colptr, pairs), _canonical(ref_colptr, ref_pairs)), f"call {call}: pairs differ"
        assert int(bad) == 0


def test_noalloc_csc_with_no_pairs_gives_zero_offsets():
    lib, fn = _lib()
    # a previous call leaves counts in the shared scratch; this call must not see them
    vals, idx = _random_selection(64, 8, 4096, 3)
    assert _call(fn, vals, idx, 4096)[0] == 0
    empty_v = torch.empty(0, device="cuda")
    empty_i = torch.empty(0, dtype=torch.int32, device="cuda")
    rc, colptr, _ = _call(fn, empty_v, empty_i, 4096)
    assert rc == 0, lib.sb_noalloc_strerror(rc)
    assert torch.equal(colptr, torch.zeros_like(colptr))


def test_noalloc_csc_skips_and_counts_out_of_range_indices():
    lib, fn = _lib()
    M, k, N = 128, 8, 2048
    vals, idx = _random_selection(M, k, N, 4)
    vals = vals.abs() + 0.1  # every in-range pair is kept
    idx[5, 0] = N
    idx[9, 2] = N + 1000
    bad = torch.zeros(1, dtype=torch.int32, device="cuda")
    rc, colptr, pairs = _call(fn, vals, idx, N, bad)
    assert rc == 0, lib.sb_noalloc_strerror(rc)
    assert int(bad) == 2
    ok = idx.clone()
    ok[5, 0] = -1
    ok[9, 2] = -1
    ref_colptr, ref_pairs = _reference(vals, ok, N)
    assert torch.equal(colptr, ref_colptr)
    assert torch.equal(_canonical(colptr, pairs), _canonical(ref_colptr, ref_pairs))


def test_noalloc_csc_rejects_oversized_arguments():
    lib, fn = _lib()
    colptr = torch.zeros(4, dtype=torch.int64, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    rc = fn(0, 0, 0, (1 << 20) + 1, colptr.data_ptr(), 0, 0, stream)
    assert rc == 1
    assert b"1048576" in lib.sb_noalloc_strerror(rc)
    rc = fn(1, 1, 1 << 31, 3, colptr.data_ptr(), 1, 0, stream)  # never dereferenced: rejected first
    assert rc == 5
    assert b"2147483647" in lib.sb_noalloc_strerror(rc)
