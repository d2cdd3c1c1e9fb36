"""Host-side plan of the P2P row router: routes, destination rows, release slots and the TP-member
fan-out (every member of a consumer's SAE TP group gets its own copy and its own release flag)."""

import pytest

from saelens_b200.parallel.row_router import ROUTE_CHUNK_ROWS, route_plan
from saelens_b200.parallel.shard_routing import compute_routing_table


def _covered(plans, batch_rows, P):
    """Every producer row lands exactly once in each receiving rank's batch, producers in order."""
    got = {}
    for rank, plan in plans.items():
        for row_start, n_rows, dst, dst_row in plan.table:
            for i in range(n_rows):
                key = (dst, dst_row + i)
                assert key not in got, f"row {key} written twice"
                got[key] = (plan.p_idx, row_start + i)
    return got


@pytest.mark.parametrize("P,Q", [(1, 1), (2, 1), (1, 2), (3, 2), (4, 4), (2, 3)])
def test_default_plan_matches_routing_table(P, Q):
    producers = list(range(P))
    consumers = list(range(P, P + Q))
    batch = 48
    routes = compute_routing_table(P, Q, batch)
    plans = {rk: route_plan(producers, consumers, batch, rk) for rk in producers + consumers}
    for p in producers:
        plan = plans[p]
        mine = [r for r in routes if r.producer_idx == p]
        assert [t[:3] for t in plan.table] == [[r.row_start, r.n_rows, consumers[r.consumer_idx]] for r in mine]
        # one release flag per consumer, indexed by the consumer
        assert plan.free_slots == [r.consumer_idx for r in mine]
    got = _covered(plans, batch, P)
    for c, crank in enumerate(consumers):
        rows = [got[(crank, i)] for i in range(plans[crank].rows_for[c])]
        assert rows == sorted(rows)  # earlier producers first, rows in order
        assert plans[crank].m_slot == c
        chunks = [0] * P
        for r in routes:
            if r.consumer_idx == c:
                chunks[r.producer_idx] += -(-r.n_rows // ROUTE_CHUNK_ROWS)
        assert plans[crank].chunks == chunks
    assert sum(len(rows) for rows in [[k for k in got if k[0] == c] for c in consumers]) == P * batch


@pytest.mark.parametrize("P,Q,TP", [(1, 1, 2), (2, 2, 2), (4, 2, 2), (2, 1, 4)])
def test_member_plan_fans_out_to_every_tp_member(P, Q, TP):
    producers = list(range(P))
    consumers = [P + c * TP for c in range(Q)]
    members = [[P + c * TP + t for t in range(TP)] for c in range(Q)]
    batch = 64
    ranks = producers + [m for ms in members for m in ms]
    plans = {rk: route_plan(producers, consumers, batch, rk, members) for rk in ranks}
    default = {rk: route_plan(producers, consumers, batch, rk) for rk in producers + consumers}
    got = _covered(plans, batch, P)
    for c in range(Q):
        ref = [got[(consumers[c], i)] for i in range(plans[consumers[c]].rows_for[c])]
        for m in members[c]:
            plan = plans[m]
            assert plan.c_idx == c
            assert plan.chunks == default[consumers[c]].chunks  # each member counts its own arrivals
            # every member holds the same rows in the same order as the root
            assert [got[(m, i)] for i in range(plan.rows_for[c])] == ref
    # release slots: one per (consumer, member), distinct, and each producer waits on every member
    slots = {plans[m].m_slot for ms in members for m in ms}
    assert slots == set(range(Q * TP))
    for p in producers:
        dsts = {(t[2], s) for t, s in zip(plans[p].table, plans[p].free_slots)}
        for t, s in zip(plans[p].table, plans[p].free_slots):
            assert plans[t[2]].m_slot == s
        assert len(dsts) == len(plans[p].table)


def test_member_plan_rejects_bad_layouts():
    with pytest.raises(ValueError):  # first member must be the consumer root
        route_plan([0], [1], 8, 0, [[2, 1]])
    with pytest.raises(ValueError):  # one rank, two consumers
        route_plan([0], [1, 2], 8, 0, [[1, 3], [2, 3]])
    with pytest.raises(ValueError):  # more destinations than the kernel takes
        route_plan([0], [1, 2], 8, 0, [list(range(1, 2)) + list(range(3, 12)), [2] + list(range(12, 20))])
