"""NVLink row routing (shard routing P x Q) with fused normalisation + bf16 cast, 2 ranks."""

import math
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


def _batch(p, step, rows, d):
    g = torch.Generator().manual_seed(1000 * p + step)
    return torch.randn(rows, d, generator=g) * (1 + p)


def _worker(rank, world, port, producers, consumers, rows, d, steps, out_dir):
    import torch.distributed as dist
    from datetime import timedelta

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    from saelens_b200.parallel.row_router import P2PRowRouter

    router = P2PRowRouter(dist.group.WORLD, producers, consumers, rows, d, normalize="unit_norm",
                          scale=math.sqrt(d))
    got = []
    for step in range(steps):
        if rank in producers:
            router.send(_batch(producers.index(rank), step, rows, d).cuda())
        if rank in consumers:
            got.append(router.recv().clone().cpu())
            router.release()
    torch.cuda.synchronize()
    router.status.check("router")
    torch.save(got, os.path.join(out_dir, f"r{rank}.pt"))
    router.close()
    dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("producers,consumers", [([0], [1]), ([0, 1], [0, 1]), ([1], [0, 1])])
def test_row_router_matches_routing_table(tmp_path, producers, consumers):
    import torch.multiprocessing as mp

    from saelens_b200.parallel.shard_routing import compute_routing_table

    rows, d, steps = 200, 384, 5
    mp.spawn(_worker, args=(2, _free_port(), producers, consumers, rows, d, steps, str(tmp_path)), nprocs=2,
             join=True)
    routes = compute_routing_table(len(producers), len(consumers), rows)
    for ci, c in enumerate(consumers):
        got = torch.load(tmp_path / f"r{c}.pt")
        assert len(got) == steps
        for step in range(steps):
            parts = []
            for r in sorted([r for r in routes if r.consumer_idx == ci], key=lambda r: r.producer_idx):
                x = _batch(r.producer_idx, step, rows, d)[r.row_start : r.row_end]
                parts.append((x / x.norm(dim=-1, keepdim=True) * math.sqrt(d)).to(torch.bfloat16))
            want = torch.cat(parts)
            assert got[step].shape == want.shape
            assert torch.allclose(got[step].float(), want.float(), atol=2e-2, rtol=2e-2), (c, step)
