"""The page-locked host ring on a GPU: a producer copies device rows straight into its slots, the
trainer-side provider copies claimed slots straight to the device on a side stream; the rows it
serves equal the rows written (the same as the pageable staging path), and every slot is FREE
again after it was read."""

import os
import shutil
import uuid

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture
def shm_dir():
    """A directory on /dev/shm (tmpfs, where the ring lives in real runs and can be page-locked)."""
    d = os.path.join("/dev/shm", f"sb_ring_test_{uuid.uuid4().hex[:8]}")
    os.makedirs(d)
    yield d
    shutil.rmtree(d, ignore_errors=True)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_registered_ring_round_trip(shm_dir, dtype):
    from saelens_b200.training.shared_activation_buffer import ChunkState, SharedActivationBuffer
    from saelens_b200.training.streaming_activation_provider import StreamingActivationProvider

    T, D, n_chunks = 256, 128, 3
    kw = dict(name="ring_gpu", num_chunks=4, chunk_size_tokens=T, d_model=D, num_producers=1,
              target_chunks=n_chunks, base_dir=shm_dir)
    prod = SharedActivationBuffer(create=True, dtype=dtype, **kw)
    cons = SharedActivationBuffer(create=False, **kw)
    assert prod.register_for_device_copies() and cons.register_for_device_copies()
    g = torch.Generator(device="cuda").manual_seed(0)
    rows = [torch.randn(T, D, device="cuda", generator=g).to(dtype) for _ in range(n_chunks)]
    for r in rows:
        idx, _ = prod.allocate_write_chunk()
        prod.write_chunk(idx, r, T)  # device tensor -> page-locked slot
        prod.mark_ready(idx)
    prod.signal_done()
    prov = StreamingActivationProvider(cons, T, prefetch_chunks=2, device="cuda", d_model=D, dtype=dtype,
                                       shuffle=False, random_chunks=False)
    assert prov._direct
    got = []
    while True:
        try:
            got.append(next(prov))
        except StopIteration:
            break
    torch.cuda.synchronize()
    out = torch.cat(got)
    assert out.shape == (n_chunks * T, D) and out.dtype == dtype
    assert torch.equal(out, torch.cat(rows))  # slots claimed in slot order, no shuffle
    assert all(int(cons._slots[i, 0]) == ChunkState.FREE for i in range(4))
    cons.close()
    prod.close()


def test_refused_registration_keeps_the_staging_path(tmp_path):
    """Whether or not the driver pins a ring mapped from a disk file, the answer leaves no CUDA
    error pending, and an unregistered ring still serves its rows (staging-copy path)."""
    from saelens_b200.training.shared_activation_buffer import SharedActivationBuffer
    from saelens_b200.training.streaming_activation_provider import StreamingActivationProvider

    kw = dict(name="ring_disk", num_chunks=2, chunk_size_tokens=64, d_model=32, num_producers=1, target_chunks=1,
              base_dir=str(tmp_path))
    buf = SharedActivationBuffer(create=True, dtype=torch.float32, **kw)
    buf.register_for_device_copies()
    torch.zeros(1, device="cuda").add_(1)  # a launch: would raise if an error were left pending
    torch.cuda.synchronize()
    cons = SharedActivationBuffer(create=False, **kw)
    rows = torch.randn(64, 32)
    idx, _ = buf.allocate_write_chunk()
    buf.write_chunk(idx, rows, 64)
    buf.mark_ready(idx)
    buf.signal_done()
    prov = StreamingActivationProvider(cons, 64, prefetch_chunks=1, device="cuda", d_model=32, shuffle=False,
                                       random_chunks=False)
    assert torch.equal(next(prov).cpu(), rows)
    cons.close()
    buf.close()


def test_shuffled_refill_gathers_pool_and_new_rows_in_one_pass(shm_dir, monkeypatch):
    """With shuffle on, a CUDA refill serves the leftover pool rows followed by the new rows in a
    random order through the native two-source gather; the same generator seed gives the same
    stream as the concatenate-then-index formulation, and every written row is served once."""
    from saelens_b200 import ops
    from saelens_b200.training.shared_activation_buffer import SharedActivationBuffer
    from saelens_b200.training.streaming_activation_provider import StreamingActivationProvider

    T, D, n_chunks, batch = 256, 64, 5, 96  # batch does not divide a chunk: refills keep leftovers
    g = torch.Generator(device="cuda").manual_seed(3)
    rows = [torch.randn(T, D, device="cuda", generator=g) for _ in range(n_chunks)]

    def serve(name):
        kw = dict(name=name, num_chunks=8, chunk_size_tokens=T, d_model=D, num_producers=1,
                  target_chunks=n_chunks, base_dir=shm_dir)
        prod = SharedActivationBuffer(create=True, dtype=torch.float32, **kw)
        cons = SharedActivationBuffer(create=False, **kw)
        for r in rows:
            idx, _ = prod.allocate_write_chunk()
            prod.write_chunk(idx, r.cpu(), T)
            prod.mark_ready(idx)
        prod.signal_done()
        prov = StreamingActivationProvider(cons, batch, prefetch_chunks=2, device="cuda", d_model=D,
                                           shuffle=True, random_chunks=False,
                                           generator=torch.Generator(device="cuda").manual_seed(11))
        got = []
        while True:
            try:
                got.append(next(prov))
            except StopIteration:
                break
        cons.close()
        prod.close()
        return torch.cat(got)

    native = serve("ring_shuffle_a")

    def torch_gather(a, b=None, perm=None, out=None):
        src = a if b is None else torch.cat([a, b])
        return src[perm] if perm is not None else src.clone()

    monkeypatch.setattr(ops, "gather_rows", torch_gather)
    reference = serve("ring_shuffle_b")
    assert torch.equal(native, reference)
    served = native.shape[0]
    allrows = torch.cat(rows)
    # every served row is one of the written rows, and no written row is served twice
    d = torch.cdist(native, allrows, compute_mode="donot_use_mm_for_euclid_dist")
    assert bool((d.min(dim=1).values == 0).all())
    assert int(d.argmin(dim=1).unique().numel()) == served
