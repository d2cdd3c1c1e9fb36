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
                   ctypes.c_void_p, ctypes.c_void_p]
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


def test_noalloc_csc_matches_allocating_path_twice():
    lib, fn = _lib()
    M, k, N = 1024, 32, 8192
    for call, seed in enumerate((1, 2)):  # two calls in a row: the shared scratch is reused
        vals, idx = _random_selection(M, k, N, seed)
        ref_colptr, ref_pairs = _reference(vals, idx, N)
        colptr = torch.full((N + 1,), -5, dtype=torch.int64, device="cuda")
        pairs = torch.full((M * k,), -5, dtype=torch.int64, device="cuda")
        rc = fn(vals.data_ptr(), idx.data_ptr(), M * k, N, colptr.data_ptr(), pairs.data_ptr(),
                torch.cuda.current_stream().cuda_stream)
        torch.cuda.synchronize()
        assert rc == 0, lib.sb_noalloc_strerror(rc)
        assert torch.equal(colptr, ref_colptr), f"call {call}: colptr differs"
        assert torch.equal(_canonical(colptr, pairs), _canonical(ref_colptr, ref_pairs)), f"call {call}: pairs differ"


def test_noalloc_csc_rejects_oversized_latent_count():
    lib, fn = _lib()
    colptr = torch.zeros(4, dtype=torch.int64, device="cuda")
    rc = fn(0, 0, 0, (1 << 20) + 1, colptr.data_ptr(), 0, torch.cuda.current_stream().cuda_stream)
    assert rc == 1
    assert b"1048576" in lib.sb_noalloc_strerror(rc)
