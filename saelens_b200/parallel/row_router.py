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

from typing import Sequence

import torch
import torch.distributed as dist

from saelens_b200.parallel.shard_routing import compute_routing_table, rows_per_consumer
from saelens_b200.parallel.symm_heap import SymmetricHeap, slab_bytes_needed

ROUTE_CHUNK_ROWS = 8  # rows per published chunk; the kernel's RT_RR
_MODES = {"none": 0, "scale": 1, "unit_norm": 2}


class P2PRowRouter:
    def __init__(self, group: dist.ProcessGroup | None, producer_ranks: Sequence[int],
                 consumer_ranks: Sequence[int], batch_rows: int, d: int, normalize: str = "none",
                 scale: float = 1.0):
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
        self.routes = compute_routing_table(self.P, self.Q, batch_rows)
        self.rows_for = rows_per_consumer(self.routes, self.Q)
        self.rows_cap = max(self.rows_for)
        sizes = [2 * self.rows_cap * self.d * 2, self.P * 4, self.Q * 4]
        self.heap = SymmetricHeap(group, slab_bytes_needed(sizes) + 4096)
        self.land = self.heap.alloc((2, self.rows_cap, self.d), torch.bfloat16)
        self.cnt = self.heap.alloc(max(self.P, 1), torch.int32)
        self.free = self.heap.alloc(max(self.Q, 1), torch.int32)
        self.land_local = self.heap.local(self.land)
        self.cnt_local = self.heap.local(self.cnt)
        self.status = StatusWord(self.heap.device)
        # destination row of producer p's block inside consumer c's batch: earlier producers first
        offset: dict[tuple[int, int], int] = {}
        fill = [0] * self.Q
        for r in sorted(self.routes, key=lambda r: (r.consumer_idx, r.producer_idx)):
            offset[(r.producer_idx, r.consumer_idx)] = fill[r.consumer_idx]
            fill[r.consumer_idx] += r.n_rows
        self.p_idx = self.producers.index(self.rank) if self.rank in self.producers else None
        self.c_idx = self.consumers.index(self.rank) if self.rank in self.consumers else None
        if self.p_idx is not None:
            mine = [r for r in self.routes if r.producer_idx == self.p_idx]
            self.table = torch.tensor([[r.row_start, r.n_rows, self.consumers[r.consumer_idx],
                                        offset[(r.producer_idx, r.consumer_idx)]] for r in mine], dtype=torch.int64)
            self.free_slots = [r.consumer_idx for r in mine]
        if self.c_idx is not None:
            chunks = [0] * self.P
            for r in self.routes:
                if r.consumer_idx == self.c_idx:
                    chunks[r.producer_idx] += (r.n_rows + ROUTE_CHUNK_ROWS - 1) // ROUTE_CHUNK_ROWS
            self._chunks = torch.tensor(chunks, dtype=torch.int64, device=self.heap.device)
            self._producer_mask = 0
            for p in self.producers:
                self._producer_mask |= 1 << p
        self.send_epoch = 0
        self.recv_epoch = 0

    @staticmethod
    def _host_wait(view: torch.Tensor, target: torch.Tensor, timeout_s: float, what: str) -> None:
        """Poll device words from the host until view >= target (elementwise): long waits (an LM
        step, a slow consumer) happen here, so the kernels' own bounded waits find the data."""
        t0 = time.monotonic()
        while True:
            if bool((view.to(torch.int64).cpu() >= target).all()):
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
            free = self.heap.local(self.free)[torch.tensor(self.free_slots, device=self.heap.device)]
            self._host_wait(free, torch.tensor(self.send_epoch + 1 - 2), host_wait_s, "consumer release")
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
            self._host_wait(self.cnt_local[: self.P], targets.cpu(), host_wait_s, "producer rows")
        self.nat.p2p_wait_targets(self.cnt_local, targets, self.status.tensor)
        return self.land_local[(self.recv_epoch - 1) % 2, : self.rows_for[self.c_idx]]

    def release(self) -> None:
        """Consumer: the last received slot may be overwritten (stream-ordered)."""
        self.nat.p2p_signal(self.heap.bases, self.rank, self.free.offset, self.c_idx, self._producer_mask,
                            self.recv_epoch)

    def close(self) -> None:
        self.heap.close()
