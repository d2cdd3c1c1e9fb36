"""Device activation ring over NVLink (2 ranks: producer GPU 0, consumer GPU 1): chunks arrive
normalised and cast, a full ring makes the producer wait, and a consumer waiting on an empty ring
gets a TimeoutError from the bounded device wait (nothing hangs)."""

import math
import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu

D, ROWS, N_CHUNKS = 512, 256, 8


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _chunk(i):
    rows = ROWS - 56 if i == N_CHUNKS - 1 else ROWS
    return torch.randn(rows, D, generator=torch.Generator().manual_seed(100 + i))


def _worker(rank, world, port, out_dir):
    import torch.distributed as dist
    from datetime import timedelta

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    from saelens_b200.parallel.device_ring import DeviceActivationRing

    ring = DeviceActivationRing(dist.group.WORLD, [0], 1, n_slots=3, chunk_rows=ROWS, d=D, normalize="unit_norm",
                                scale=math.sqrt(D), header_path=os.path.join(out_dir, "ring_header"),
                                claim_timeout_ms=500.0)
    res = {}
    if rank == 0:
        for i in range(N_CHUNKS):
            ring.write(_chunk(i).cuda(), timeout_s=60.0)
        ring.producer_done()
    else:
        got = []
        for _ in range(N_CHUNKS):
            out, rows = ring.take(timeout_s=60.0)
            got.append(out[:rows].float().cpu())
        res["got"] = got
        res["done"] = ring.producers_done()
        try:
            ring.take(timeout_s=1.0)
            res["timed_out"] = False
        except TimeoutError:
            res["timed_out"] = True
        res["ready_after"] = ring.ready_chunks()
    dist.barrier()
    if rank == 1:
        res["header"] = ring.header.snapshot()
        torch.save(res, os.path.join(out_dir, "consumer.pt"))
    ring.close()
    dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_device_ring_producer_to_consumer(tmp_path):
    import torch.multiprocessing as mp

    mp.spawn(_worker, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True)
    res = torch.load(tmp_path / "consumer.pt")
    want = []
    for i in range(N_CHUNKS):
        x = _chunk(i)
        want.append((x / x.norm(dim=-1, keepdim=True) * math.sqrt(D)).to(torch.bfloat16).float())
    used = set()
    for g in res["got"]:
        match = [i for i, w in enumerate(want) if i not in used and w.shape == g.shape
                 and torch.allclose(g, w, atol=2e-2, rtol=1e-2)]
        assert match, "a received chunk matches no sent chunk"
        used.add(match[0])
    assert used == set(range(N_CHUNKS))
    assert res["done"] and res["timed_out"] and res["ready_after"] == 0
    assert res["header"]["written"] == [N_CHUNKS, 0] and res["header"]["taken"] == [0, N_CHUNKS]
    assert res["header"]["done"] == [1, 0]
