"""Peer-memory kernels: bounded flag waits, the two-shot NVLink all-reduce (2 ranks)."""

import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


@pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a GPU")
def test_flag_wait_gives_up_with_status():
    """A flag that nothing sets: the wait ends after its time limit with status 5 and the context
    stays usable."""
    from saelens_b200.ops import native
    from saelens_b200.ops.status import KernelTimeoutError, StatusWord

    nat = native()
    st = StatusWord("cuda")
    flags = torch.zeros(4, dtype=torch.int32, device="cuda")
    nat.p2p_wait_flags(flags, 1, st.tensor)
    torch.cuda.synchronize()
    assert st.code() == 5
    with pytest.raises(KernelTimeoutError):
        st.check("wait")
    flags.fill_(3)
    nat.p2p_wait_flags(flags, 2, st.tensor)  # already satisfied
    torch.cuda.synchronize()
    assert st.code() == 0
    assert float(torch.ones(8, device="cuda").sum()) == 8.0


def _ar_worker(rank, world, port, out_dir):
    import torch.distributed as dist
    from datetime import timedelta

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    from saelens_b200.ops import native
    from saelens_b200.ops.status import StatusWord
    from saelens_b200.parallel.symm_heap import SymmetricHeap
    from saelens_b200.parallel.tp_engine import _AllReduceBufs

    nat = native()
    heap = SymmetricHeap(dist.group.WORLD, 64 << 20)
    st = StatusWord("cuda")
    tk = torch.zeros(1, dtype=torch.int32, device="cuda")
    results = {}
    for name, n, dtype, scale in (("f32_small", 8195, torch.float32, 1.0), ("bf16_big", (1 << 20) + 24,
                                                                              torch.bfloat16, 0.5)):
        bufs = _AllReduceBufs(heap, nat, n, dtype)
        outs = []
        for ep in range(1, 4):
            g = torch.Generator(device="cpu").manual_seed(100 * ep + rank)
            x = torch.randn(n, generator=g).to(dtype).cuda()
            nat.p2p_allreduce(x, scale, heap.bases, rank, bufs.land, bufs.cnt, bufs.out_buf.offset, bufs.flag, ep,
                              tk, st.tensor)
            outs.append(bufs.out.clone().cpu())
        results[name] = outs
    # exact int32 sums (histograms, counts) above 2^24, where fp32 accumulation would round
    bufs = _AllReduceBufs(heap, nat, 65536 + 7, torch.int32)
    xi = (torch.arange(65536 + 7, dtype=torch.int64) * (rank + 3) + (1 << 24) + 1).to(torch.int32).cuda()
    nat.p2p_allreduce(xi, 1.0, heap.bases, rank, bufs.land, bufs.cnt, bufs.out_buf.offset, bufs.flag, 1, tk,
                      st.tensor)
    results["i32"] = bufs.out.clone().cpu()
    torch.cuda.synchronize()
    st.check("allreduce")
    torch.save(results, os.path.join(out_dir, f"ar{rank}.pt"))
    heap.close()
    dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_p2p_allreduce_two_ranks(tmp_path):
    import torch.multiprocessing as mp

    mp.spawn(_ar_worker, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True)
    res = [torch.load(tmp_path / f"ar{r}.pt") for r in range(2)]
    for name, n, dtype, scale in (("f32_small", 8195, torch.float32, 1.0), ("bf16_big", (1 << 20) + 24,
                                                                            torch.bfloat16, 0.5)):
        for ep in range(1, 4):
            xs = [torch.randn(n, generator=torch.Generator().manual_seed(100 * ep + r)).to(dtype).float()
                  for r in range(2)]
            want = (xs[0] + xs[1]) * scale
            for r in range(2):
                got = res[r][name][ep - 1].float()
                tol = 1e-6 if dtype == torch.float32 else 1e-2
                assert torch.allclose(got, want.to(dtype).float(), atol=tol, rtol=tol), (name, ep, r)
            assert torch.equal(res[0][name][ep - 1], res[1][name][ep - 1])
    ar = torch.arange(65536 + 7, dtype=torch.int64)
    want_i = (ar * 3 + (1 << 24) + 1) + (ar * 4 + (1 << 24) + 1)
    for r in range(2):
        assert torch.equal(res[r]["i32"].to(torch.int64), want_i)
