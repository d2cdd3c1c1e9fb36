"""P-producer x Q-consumer row routing (the table sae_lens/shard_routing.py:31-89 defines).

Producer p owns [p/P, (p+1)/P) of the unit interval and consumer c owns [c/Q, (c+1)/Q).  In
units of 1/(P*Q) those are [p*Q, (p+1)*Q) and [c*P, (c+1)*P).  Every overlapping pair is an
edge; producer p's `batch_size` rows are split over its edges in proportion to the overlap,
the last edge taking the integer remainder.  Producers and consumers compute the table
independently and must agree row for row, so the arithmetic is the reference's exactly.
"""

from __future__ import annotations

from dataclasses import dataclass


@dataclass(frozen=True)
class ShardRoute:
    producer_idx: int
    consumer_idx: int
    row_start: int  # inclusive, in producer p's batch
    row_end: int    # exclusive

    @property
    def n_rows(self) -> int:
        return self.row_end - self.row_start


def compute_routing_table(P: int, Q: int, batch_size: int) -> list[ShardRoute]:
    if P < 1 or Q < 1:
        raise ValueError(f"P and Q must be >= 1, got P={P}, Q={Q}")
    if batch_size < 1:
        raise ValueError(f"batch_size must be >= 1, got {batch_size}")
    out: list[ShardRoute] = []
    for p in range(P):
        lo, hi = p * Q, (p + 1) * Q
        edges = [(c, min(hi, (c + 1) * P) - max(lo, c * P)) for c in range(Q)]
        edges = [(c, ov) for c, ov in edges if ov > 0]
        start = 0
        for i, (c, ov) in enumerate(edges):
            n = (ov * batch_size) // Q if i < len(edges) - 1 else batch_size - start
            if n == 0:
                raise ValueError(
                    f"routing {batch_size} rows per producer is too small for {P} producers and {Q} consumers: "
                    f"producer {p} shares {ov} / {Q} of its rows with consumer {c}, which rounds to no rows"
                )
            out.append(ShardRoute(p, c, start, start + n))
            start += n
        if start != batch_size:
            raise AssertionError(f"producer {p} assigned {start} rows, expected {batch_size}")
    return out


def routes_for_producer(routes: list[ShardRoute], p: int) -> list[ShardRoute]:
    return [r for r in routes if r.producer_idx == p]


def routes_for_consumer(routes: list[ShardRoute], c: int) -> list[ShardRoute]:
    return [r for r in routes if r.consumer_idx == c]


def rows_per_consumer(routes: list[ShardRoute], Q: int) -> list[int]:
    """Rows each consumer receives per producer step (sum over its incoming routes)."""
    out = [0] * Q
    for r in routes:
        out[r.consumer_idx] += r.n_rows
    return out
