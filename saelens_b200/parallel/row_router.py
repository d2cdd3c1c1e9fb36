"""Producer -> consumer activation routing over NVLink (shard routing P x Q, peer-memory kernel).

The routing table is the interval-overlap table of `shard_routing.compute_routing_table`: producer
p's `batch_rows` rows are split over the consumers whose unit-interval share overlaps its own.
Instead of one NCCL send/recv pair per route plus separate cast and normalisation passes
(sae_lens/training/activations_store.py:1482-1606), one kernel per producer step writes every
route's rows straight into the consumers' landing buffers (NVSwitch P2P stores), converting to
bf16 and applying the activation normalisation on the way, and counts the arrived chunks on the
consumer.  Consumers see their rows ordered by producer index (the assembled batch order).

Landing buffers are double-buffered: the producer's kernel for step e waits (bounded) until every
destination consumer has released step e - 2, so a slow consumer throttles the producers instead
of being overwritten.

All ranks of `group` construct the router (collective); a rank may be a producer, a consumer,
both or neither.
"""

from __future__ import annotations

import time
from dataclasses import dataclass, field
from typing import Callable, Sequence

import torch
import torch.distributed as dist

from saelens_b200.parallel.shard_routing import compute_routing_table, rows_per_consumer
from saelens_b200.parallel.symm_heap import SymmetricHeap, slab_bytes_needed

ROUTE_CHUNK_ROWS = 8  # rows per published chunk; the kernel's RT_RR
_MODES = {"none": 0, "scale": 1, "unit_norm": 2}


@dataclass
class RoutePlan:
    """Host-side plan of one rank in the router (no device state)."""

    routes: list
    rows_for: list[int]
    members: list[list[int]]
    member_slot: dict[tuple[int, int], int]  # (consumer, receiving rank) -> release flag index
    p_idx: int | None
    c_idx: int | None
    m_slot: int | None
    table: list[list[int]] = field(default_factory=list)  # [row_start, n_rows, dst_rank, dst_row]
    free_slots: list[int] = field(default_factory=list)
    chunks: list[int] = field(default_factory=list)  # chunks expected from each producer


def route_plan(producers: Sequence[int], consumers: Sequence[int], batch_rows: int, rank: int,
               consumer_members: Sequence[Sequence[int]] | None = None) -> RoutePlan:
    """Routes, destination rows and release slots for `rank`.  `consumer_members[c]` (first entry
    `consumers[c]`) lists every rank that receives consumer c's rows; each gets its own copy of the
    rows and its own release flag."""
    P, Q = len(producers), len(consumers)
    routes = compute_routing_table(P, Q, batch_rows)
    members = [list(m) for m in consumer_members] if consumer_members is not None else [[c] for c in consumers]
    if len(members) != Q or any(not members[c] or members[c][0] != consumers[c] for c in range(Q)):
        raise ValueError("consumer_members[c] must start with consumer_ranks[c]")
    member_slot: dict[tuple[int, int], int] = {}
    for c, ranks in enumerate(members):
        for rk in ranks:
            if any(rk == r for (_, r) in member_slot):
                raise ValueError(f"rank {rk} receives rows for more than one consumer")
            member_slot[(c, rk)] = len(member_slot)
    # destination row of producer p's block inside consumer c's batch: earlier producers first
    offset: dict[tuple[int, int], int] = {}
    fill = [0] * Q
    for r in sorted(routes, key=lambda r: (r.consumer_idx, r.producer_idx)):
        offset[(r.producer_idx, r.consumer_idx)] = fill[r.consumer_idx]
        fill[r.consumer_idx] += r.n_rows
    p_idx = producers.index(rank) if rank in producers else None
    c_idx = next((c for c, ranks in enumerate(members) if rank in ranks), None)
    plan = RoutePlan(routes, rows_per_consumer(routes, Q), members, member_slot, p_idx, c_idx,
                     member_slot[(c_idx, rank)] if c_idx is not None else None)
    if p_idx is not None:
        for r in routes:
            if r.producer_idx != p_idx:
                continue
            for rk in members[r.consumer_idx]:
                plan.table.append([r.row_start, r.n_rows, rk, offset[(r.producer_idx, r.consumer_idx)]])
                plan.free_slots.append(member_slot[(r.consumer_idx, rk)])
        if len(plan.table) > 16:  # the kernel's RT_MAX_ROUTES
            raise ValueError(f"producer {p_idx} has {len(plan.table)} destinations; at most 16 are supported")
    if c_idx is not None:
        plan.chunks = [0] * P
        for r in routes:
            if r.consumer_idx == c_idx:
                plan.chunks[r.producer_idx] += (r.n_rows + ROUTE_CHUNK_ROWS - 1) // ROUTE_CHUNK_ROWS
    return plan


class P2PRowRouter:
    def __init__(self, group: dist.ProcessGroup | None, producer_ranks: Sequence[int],
                 consumer_ranks: Sequence[int], batch_rows: int, d: int, normalize: str = "none",
                 scale: float = 1.0, consumer_members: Sequence[Sequence[int]] | None = None):
        """`consumer_members[c]` lists every rank that receives consumer c's rows (an SAE TP
        group with replicated input): the producer stores the rows into each member's landing
        buffer directly, so no broadcast follows.  Default: the consumer rank alone."""
        from saelens_b200.ops import native
        from saelens_b200.ops.status import StatusWord

        if normalize not in _MODES:
            raise ValueError(f"normalize must be one of {sorted(_MODES)}")
        self.nat = native()
        self.group = group
        self.rank = dist.get_rank(group)
        self.producers = list(producer_ranks)
        self.consumers = list(consumer_ranks)
        self.P, self.Q = len(self.producers), len(self.consumers)
        self.d = int(d)
        self.mode = _MODES[normalize]
        self.scale = float(scale)
        plan = route_plan(self.producers, self.consumers, batch_rows, self.rank, consumer_members)
        self.routes, self.rows_for, self.members = plan.routes, plan.rows_for, plan.members
        self.member_slot, self.p_idx, self.c_idx, self.m_slot = plan.member_slot, plan.p_idx, plan.c_idx, plan.m_slot
        self.rows_cap = max(self.rows_for)
        n_slots = len(self.member_slot)
        sizes = [2 * self.rows_cap * self.d * 2, self.P * 4, n_slots * 4]
        self.heap = SymmetricHeap(group, slab_bytes_needed(sizes) + 4096)
        self.land = self.heap.alloc((2, self.rows_cap, self.d), torch.bfloat16)
        self.cnt = self.heap.alloc(max(self.P, 1), torch.int32)
        self.free = self.heap.alloc(max(n_slots, 1), torch.int32)
        self.land_local = self.heap.local(self.land)
        self.cnt_local = self.heap.local(self.cnt)
        self.status = StatusWord(self.heap.device)
        if self.p_idx is not None:
            self.table = torch.tensor(plan.table, dtype=torch.int64).reshape(-1, 4)
            self.free_slots = plan.free_slots
        if self.c_idx is not None:
            self._chunks = torch.tensor(plan.chunks, dtype=torch.int64, device=self.heap.device)
            self._producer_mask = 0
            for p in self.producers:
                self._producer_mask |= 1 << p
        self.send_epoch = 0
        self.recv_epoch = 0

    @staticmethod
    def _host_wait(read: Callable[[], torch.Tensor], target: torch.Tensor, timeout_s: float, what: str) -> None:
        """Poll device words from the host until read() >= target (elementwise): long waits (an LM
        step, a slow consumer) happen here, so the kernels' own bounded waits find the data.
        `read` reads the words afresh at every poll."""
        t0 = time.monotonic()
        while True:
            if bool((read().to(torch.int64).cpu() >= target).all()):
                return
            if time.monotonic() - t0 > timeout_s:
                raise TimeoutError(f"row router: {what} not reached within {timeout_s:.0f} s")
            time.sleep(5e-5)

    def send(self, acts: torch.Tensor, host_wait_s: float | None = None) -> None:
        """Producer: route this step's rows (fp32 or bf16 [batch_rows, d]) to the consumers.
        With `host_wait_s`, first wait on the host until the destination slots were released."""
        if self.p_idx is None:
            raise RuntimeError(f"rank {self.rank} is not a producer")
        if host_wait_s is not None and self.send_epoch + 1 >= 3:
            free = self.heap.local(self.free)
            slots = torch.tensor(self.free_slots, device=self.heap.device)
            # index inside the poll: advanced indexing copies, and a copy would never change
            self._host_wait(lambda: free[slots], torch.tensor(self.send_epoch + 1 - 2), host_wait_s,
                            "consumer release")
        self.send_epoch += 1
        self.nat.p2p_route_rows(acts, self.table, self.heap.bases, self.rank, self.land.offset, self.rows_cap,
                                (self.send_epoch - 1) % 2, self.cnt.offset, self.p_idx, self.free.offset,
                                self.free_slots, self.mode, self.scale, self.send_epoch, self.status.tensor)

    def recv(self, host_wait_s: float | None = None) -> torch.Tensor:
        """Consumer: wait (on the stream) for this step's rows; returns a view of the landing slot.
        Call `release()` once the rows have been consumed.  With `host_wait_s`, first wait on the
        host until every producer's rows arrived."""
        if self.c_idx is None:
            raise RuntimeError(f"rank {self.rank} is not a consumer")
        self.recv_epoch += 1
        targets = self._chunks * self.recv_epoch
        if host_wait_s is not None:
            self._host_wait(lambda: self.cnt_local[: self.P], targets.cpu(), host_wait_s, "producer rows")
        self.nat.p2p_wait_targets(self.cnt_local, targets, self.status.tensor)
        return self.land_local[(self.recv_epoch - 1) % 2, : self.rows_for[self.c_idx]]

    def release(self) -> None:
        """Consumer: the last received slot may be overwritten (stream-ordered)."""
        self.nat.p2p_signal(self.heap.bases, self.rank, self.free.offset, self.m_slot, self._producer_mask,
                            self.recv_epoch)

    def close(self) -> None:
        self.heap.close()
