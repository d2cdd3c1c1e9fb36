"""Shard routing table (interface of sae_lens/shard_routing.py; cases follow
tests/test_shard_routing.py)."""

import pytest

from saelens_b200.parallel.shard_routing import (
    ShardRoute,
    compute_routing_table,
    routes_for_consumer,
    routes_for_producer,
    rows_per_consumer,
)


def _partition_ok(routes, P, Q, B):
    assert {r.producer_idx for r in routes} == set(range(P))
    assert {r.consumer_idx for r in routes} == set(range(Q))
    for p in range(P):
        cur = 0
        for r in sorted(routes_for_producer(routes, p), key=lambda r: r.row_start):
            assert r.row_start == cur and r.row_end > r.row_start
            cur = r.row_end
        assert cur == B


def test_1_1():
    routes = compute_routing_table(1, 1, 10)
    assert routes == [ShardRoute(0, 0, 0, 10)]


def test_fan_in_3_1_and_fan_out_1_3():
    routes = compute_routing_table(3, 1, 12)
    assert all(r.consumer_idx == 0 and (r.row_start, r.row_end) == (0, 12) for r in routes)
    routes = compute_routing_table(1, 3, 12)
    assert len(routes) == 3 and all(r.producer_idx == 0 for r in routes)
    _partition_ok(routes, 1, 3, 12)


def test_matched_3_3_and_exact_fan_in_6_2():
    assert all(r.producer_idx == r.consumer_idx for r in compute_routing_table(3, 3, 10))
    routes = compute_routing_table(6, 2, 12)
    assert {r.producer_idx for r in routes_for_consumer(routes, 0)} == {0, 1, 2}
    assert {r.producer_idx for r in routes_for_consumer(routes, 1)} == {3, 4, 5}


def test_2_3_fan_out_overlaps():
    routes = compute_routing_table(2, 3, 12)
    assert {r.consumer_idx for r in routes_for_producer(routes, 0)} == {0, 1}
    assert {r.consumer_idx for r in routes_for_producer(routes, 1)} == {1, 2}
    assert {r.producer_idx for r in routes_for_consumer(routes, 1)} == {0, 1}


@pytest.mark.parametrize("P,Q,B", [(5, 3, 15), (4, 3, 100), (3, 4, 100), (7, 5, 100), (5, 7, 100), (2, 3, 120),
                                   (7, 4, 120), (1, 100, 200)])
def test_partition_invariants(P, Q, B):
    routes = compute_routing_table(P, Q, B)
    _partition_ok(routes, P, Q, B)
    assert sum(r.row_end - r.row_start for r in routes) == P * B
    assert sum(rows_per_consumer(routes, Q)) == P * B


@pytest.mark.parametrize("P,Q,B", [(2, 3, 1), (1, 100, 10)])
def test_zero_row_edge_raises(P, Q, B):
    with pytest.raises(ValueError, match="too small"):
        compute_routing_table(P, Q, B)
