"""Rank layouts for every topology (pure arithmetic), routing-table invariants, and real group
creation on gloo ranks."""

import os
import socket
from datetime import timedelta
from unittest import mock

import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

from saelens_b200.parallel.layout import prefix_layout, routed_layout
from saelens_b200.parallel.shard_routing import (
    compute_routing_table,
    routes_for_consumer,
    routes_for_producer,
    rows_per_consumer,
)


def test_local_overlap_prefix_groups():
    lay = prefix_layout(world_size=4, sae_tp_size=2, vllm_tp_size=4)
    assert lay.mode == "local_overlap"
    assert [r.sae_active for r in lay.roles] == [True, True, False, False]
    assert lay.group_of("sae_tp", 1) == [0, 1]
    assert lay.group_of("vllm_tp", 3) == [0, 1, 2, 3]


def test_matched_dp_layout():
    lay = prefix_layout(world_size=8, sae_tp_size=2, sae_dp_size=2, vllm_tp_size=4, vllm_dp_size=2)
    assert lay.mode == "matched_dp"
    assert lay.group_of("sae_dp", 5) == [1, 5]
    assert lay.role(6).vllm_dp_rank == 1 and lay.role(6).sae_dp_rank == 1
    assert lay.group_of("sae_tp", 4) == [4, 5]


def test_fan_in_layout_m_to_1_and_mn_to_m():
    lay = prefix_layout(world_size=4, sae_tp_size=1, sae_dp_size=1, vllm_tp_size=1, vllm_dp_size=4)
    assert lay.mode == "vllm_dp_fan_in"
    assert [r.vllm_dp_rank for r in lay.roles] == [0, 1, 2, 3]
    assert [r.sae_active for r in lay.roles] == [True, False, False, False]
    lay = prefix_layout(world_size=8, sae_tp_size=2, sae_dp_size=2, vllm_tp_size=2, vllm_dp_size=4)
    assert lay.cluster_block == 4
    assert lay.group_of("sae_dp", 1) == [1, 5]
    assert lay.role(6).vllm_dp_rank == 3 and lay.role(6).sae_dp_rank == 1


@pytest.mark.parametrize("kw", [
    dict(world_size=4, sae_dp_size=2, vllm_dp_size=1, vllm_tp_size=2, sae_tp_size=2),  # 1:m
    dict(world_size=6, sae_dp_size=2, vllm_dp_size=3),  # not multiples
    dict(world_size=5, sae_tp_size=2, vllm_tp_size=2),  # wrong world
])
def test_invalid_layouts_raise(kw):
    with pytest.raises(ValueError):
        prefix_layout(**kw)


@pytest.mark.parametrize("P,Q,B", [(1, 1, 7), (2, 3, 101), (3, 2, 64), (4, 6, 1000), (5, 5, 5)])
def test_routing_table_partitions(P, Q, B):
    table = compute_routing_table(P, Q, B)
    for p in range(P):
        rs = routes_for_producer(table, p)
        assert rs[0].row_start == 0 and rs[-1].row_end == B
        for a, b in zip(rs, rs[1:]):
            assert a.row_end == b.row_start
        assert all(r.n_rows > 0 for r in rs)
    assert sum(rows_per_consumer(table, Q)) == P * B
    for c in range(Q):
        assert routes_for_consumer(table, c), f"consumer {c} has no producer"
    with pytest.raises(ValueError):
        compute_routing_table(2, 3, 1)


def test_routing_table_matches_interval_overlap():
    # 2 producers, 3 consumers, 6 rows: p0 -> c0 (4 rows), c1 (2); p1 -> c1 (2), c2 (4)
    t = compute_routing_table(2, 3, 6)
    assert [(r.producer_idx, r.consumer_idx, r.row_start, r.row_end) for r in t] == [
        (0, 0, 0, 4), (0, 1, 4, 6), (1, 1, 0, 2), (1, 2, 2, 6)]


def test_routed_layout_overlapping_and_disjoint():
    lay = routed_layout(P=2, Q=3, vllm_tp_size=2, sae_tp_size=1, batch_size=60)
    assert lay.world_size == 4
    assert lay.roles_of(0) == {"is_producer": True, "is_consumer": True, "producer_idx": 0, "consumer_idx": 0,
                               "vllm_tp_rank": 0, "sae_tp_rank": 0}
    p2p = [g for g in lay.groups if g[0] == "consumer_p2p"]
    assert p2p[1][1] == [0, 1, 2]  # consumer 1 (rank 1) gets rows from producer roots 0 and 2
    d = routed_layout(P=2, Q=1, vllm_tp_size=2, sae_tp_size=2, batch_size=8, disjoint=True)
    assert d.world_size == 6 and d.consumer_ranks[0] == [4, 5]
    assert not d.roles_of(4)["is_producer"] and d.roles_of(4)["is_consumer"]


def test_init_distributed_creates_groups_in_layout_order():
    from saelens_b200.parallel import distributed as D

    created = []
    with mock.patch.object(dist, "is_initialized", return_value=True), \
            mock.patch.object(dist, "get_world_size", return_value=8), \
            mock.patch.object(dist, "get_rank", return_value=5), \
            mock.patch.object(dist, "new_group", side_effect=lambda ranks, backend=None: (tuple(ranks), backend)) as ng:
        D._reset()
        D.init_distributed(sae_tp_size=2, sae_dp_size=2, vllm_tp_size=4, vllm_dp_size=2)
        created = [c.args[0] for c in ng.call_args_list]
    assert created[0] == [0, 1, 2, 3]
    assert D.get_sae_tp_group()[0] == (4, 5)
    assert D.get_sae_dp_group()[0] == (1, 5)
    assert D.get_sae_tp_rank() == 1 and D.get_sae_dp_rank() == 1
    assert D.get_layout_mode() == "matched_dp"
    D._reset()


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _v2_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    from saelens_b200.parallel import distributed_v2 as V

    # overlapping 2 producers (tp 2) x 4 consumers (tp 1) on 4 ranks, all groups on gloo
    with mock.patch("saelens_b200.parallel.layout.routed_layout", wraps=routed_layout):
        lay = routed_layout(2, 4, 2, 1, 64)
        lay.groups = [(k, r, "gloo", i) for k, r, _, i in lay.groups]
        with mock.patch("saelens_b200.parallel.distributed_v2.routed_layout", return_value=lay):
            V.init_distributed_v2(2, 4, 2, 1, 64)
    import torch

    t = torch.ones(1) * (rank + 1)
    dist.all_reduce(t, group=V.get_sae_dp_group())
    q.put((rank, V.is_producer(), V.get_producer_idx(), V.get_consumer_idx(), float(t)))
    dist.barrier()
    dist.destroy_process_group()


def test_init_distributed_v2_on_gloo_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_v2_worker, args=(r, 4, _port_holder[0], q)) for r in range(4)] \
        if (_port_holder := [_port()]) else []
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=120) for _ in range(4))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert [r[2] for r in res] == [0, 0, 1, 1]
    assert [r[3] for r in res] == [0, 1, 2, 3]
    assert all(r[4] == 10.0 for r in res)  # sae_dp group = all 4 consumers: 1+2+3+4
