"""Routed exchange with uneven splits (2 producers -> 3 consumers, gloo, collective transport):
every producer row reaches exactly one consumer, each consumer gets its train batch per step,
and rows arrive in producer order."""

import os
import socket
from types import SimpleNamespace

import torch
import torch.multiprocessing as mp

P, Q, TB, D, STEPS = 2, 3, 12, 8, 3


def _port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


class _TaggedStore:
    """Batches whose first three columns are (producer, batch index, row index)."""

    def __init__(self, p: int):
        self.p, self.i = p, 0

    def __next__(self) -> torch.Tensor:
        b = torch.zeros(5, D)
        b[:, 0] = self.p
        b[:, 1] = self.i
        b[:, 2] = torch.arange(5)
        self.i += 1
        return b


def _worker(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import torch.distributed as dist

    dist.init_process_group("gloo", rank=rank, world_size=world)
    from saelens_b200.runners.routing import RoutedExchange, routing_init

    cfg = SimpleNamespace(device="cpu", train_batch_size_tokens=TB, sae=SimpleNamespace(d_in=D), dtype="float32",
                          routing_transport="collective", n_checkpoints=0, checkpoint_path=None,
                          total_training_tokens=TB * STEPS)
    runner = SimpleNamespace(cfg=cfg, vllm_dp_size=P, sae_dp_size=Q, vllm_tp_size=1, sae_tp_size=1)
    routing_init(runner)
    runner.activations_store = _TaggedStore(rank) if runner.is_route_producer else None
    ex = RoutedExchange(runner)
    got = [ex.step() for _ in range(STEPS)]
    torch.save({"role": runner.role, "got": got}, os.path.join(out, f"r{rank}.pt"))
    dist.destroy_process_group()


def test_two_producers_three_consumers(tmp_path):
    world = P + Q
    mp.spawn(_worker, args=(world, _port(), str(tmp_path)), nprocs=world, join=True)
    res = [torch.load(tmp_path / f"r{i}.pt") for i in range(world)]
    assert [r["role"] for r in res] == ["producer"] * P + ["consumer"] * Q
    for step in range(STEPS):
        ids = []
        for c in range(P, world):
            b = res[c]["got"][step]
            assert b.shape == (TB, D)  # one train batch per consumer and step
            tags = [tuple(int(v) for v in row[:3]) for row in b]
            assert [t[0] for t in tags] == sorted(t[0] for t in tags)  # producer order
            ids += tags
        assert len(ids) == len(set(ids)) == P * Q * TB // P  # no duplicates, every row delivered
    for p in range(P):
        assert all(g is None for g in res[p]["got"])
