"""Pure rank-layout arithmetic for every supported producer/trainer topology.

A layout says, for a world of ranks, which ranks form each process group and which role every
rank plays; it creates no group and needs no distributed runtime, so it can be checked for every
topology on a laptop.  `saelens_b200.parallel.distributed*` turn a layout into real
`torch.distributed` groups (every rank creating every group, in the layout's order).

Topologies (semantics of sae_lens/distributed.py:49-254 and distributed_v2.py:94-229):
* local overlap (1:1): one replica of max(vllm_tp, sae_tp) ranks; the SAE TP group and the LM TP
  group are prefixes of it.
* matched DP (m:m): `sae_dp` replicas as above, LM DP rank = SAE DP rank.
* fan-in (mn:m): `vllm_dp = n * sae_dp` LM replicas; each cluster of n LM replicas feeds one
  SAE replica (the legacy m:1 is sae_dp = 1).
* shard routing (P x Q): P producer replicas and Q consumer replicas, overlapping
  (world = max(P*vtp, Q*stp)) or disjoint (world = P*vtp + Q*stp); per-consumer P2P groups join
  the consumer's TP root with the roots of the producers routed to it.
"""

from __future__ import annotations

from dataclasses import dataclass, field

from saelens_b200.parallel.shard_routing import ShardRoute, compute_routing_table


@dataclass
class RankRole:
    rank: int
    sae_active: bool
    vllm_active: bool
    sae_tp_rank: int
    sae_dp_rank: int
    vllm_tp_rank: int
    vllm_dp_rank: int
    worker_rank: int


@dataclass
class PrefixLayout:
    """Layout of `init_distributed` (local overlap, matched DP, fan-in)."""

    mode: str
    world_size: int
    sae_tp_size: int
    sae_dp_size: int
    vllm_tp_size: int
    vllm_dp_size: int
    cluster_block: int
    worker_size: int
    # groups in creation order: (kind, ranks, backend)
    groups: list[tuple[str, list[int], str]] = field(default_factory=list)
    roles: list[RankRole] = field(default_factory=list)

    def role(self, rank: int) -> RankRole:
        return self.roles[rank]

    def group_of(self, kind: str, rank: int) -> list[int] | None:
        for k, ranks, _ in self.groups:
            if k == kind and rank in ranks:
                return ranks
        return None


def prefix_layout(world_size: int, sae_tp_size: int = 1, sae_dp_size: int = 1, vllm_tp_size: int = 1,
                  vllm_dp_size: int = 1) -> PrefixLayout:
    if sae_dp_size < 1:
        raise ValueError(f"sae_dp_size must be >= 1, got {sae_dp_size}")
    if vllm_dp_size < 1:
        raise ValueError(f"vllm_dp_size must be >= 1, got {vllm_dp_size}")
    if sae_dp_size > 1 and vllm_dp_size == 1:
        raise ValueError("sae_dp_size > 1 requires vllm_dp_size > 1; 1:m is not supported")
    if vllm_dp_size > 1 and sae_dp_size > 1:
        big, small = max(vllm_dp_size, sae_dp_size), min(vllm_dp_size, sae_dp_size)
        if big % small:
            raise ValueError("vllm_dp_size and sae_dp_size must be integer multiples of each other")
        if sae_dp_size > vllm_dp_size:
            raise ValueError("m:mn topology (sae_dp_size > vllm_dp_size) is not supported")
    fan_in = vllm_dp_size > sae_dp_size
    matched = vllm_dp_size == sae_dp_size and vllm_dp_size > 1
    if fan_in and sae_tp_size > vllm_tp_size * vllm_dp_size:
        raise ValueError("sae_tp_size > vllm_tp_size * vllm_dp_size is not supported with vllm_dp > sae_dp")
    if fan_in:
        expected = max(vllm_tp_size * vllm_dp_size, sae_tp_size * sae_dp_size)
    else:
        expected = max(vllm_tp_size, sae_tp_size) * sae_dp_size
    if world_size != expected:
        raise ValueError(
            f"world_size={world_size} != expected={expected} (vllm_tp={vllm_tp_size}, vllm_dp={vllm_dp_size}, "
            f"sae_tp={sae_tp_size}, sae_dp={sae_dp_size})"
        )
    roles: list[RankRole] = []
    groups: list[tuple[str, list[int], str]] = []
    if fan_in:
        n = vllm_dp_size // sae_dp_size
        block = max(n * vllm_tp_size, sae_tp_size)
        for r in range(world_size):
            c, w = divmod(r, block)
            sae_on = w < sae_tp_size
            vllm_on = w < n * vllm_tp_size
            roles.append(RankRole(
                rank=r, sae_active=sae_on, vllm_active=vllm_on, sae_tp_rank=w if sae_on else -1, sae_dp_rank=c,
                vllm_tp_rank=(w % vllm_tp_size) if vllm_on else -1,
                vllm_dp_rank=(c * n + w // vllm_tp_size) if vllm_on else -1,
                worker_rank=(w % vllm_tp_size) if vllm_on else -1,
            ))
        for vdp in range(vllm_dp_size):
            base = (vdp // n) * block + (vdp % n) * vllm_tp_size
            ranks = list(range(base, base + vllm_tp_size))
            groups.append(("vllm_tp", ranks, "nccl"))
            groups.append(("worker_cpu", ranks, "gloo"))
        for c in range(sae_dp_size):
            groups.append(("sae_tp", list(range(c * block, c * block + sae_tp_size)), "nccl"))
        for t in range(sae_tp_size):
            groups.append(("sae_dp", [c * block + t for c in range(sae_dp_size)], "nccl"))
        groups.append(("vllm_dp_p2p", list(range(world_size)), "gloo"))
        return PrefixLayout("vllm_dp_fan_in", world_size, sae_tp_size, sae_dp_size, vllm_tp_size, vllm_dp_size,
                            block, vllm_tp_size, groups, roles)
    rep = max(vllm_tp_size, sae_tp_size)
    for r in range(world_size):
        d, w = divmod(r, rep)
        sae_on, vllm_on = w < sae_tp_size, w < vllm_tp_size
        roles.append(RankRole(
            rank=r, sae_active=sae_on, vllm_active=vllm_on, sae_tp_rank=w if sae_on else -1, sae_dp_rank=d,
            vllm_tp_rank=w if vllm_on else -1, vllm_dp_rank=d if matched else 0, worker_rank=w,
        ))
    for d in range(sae_dp_size):
        ranks = list(range(d * rep, (d + 1) * rep))
        groups.append(("worker", ranks, "nccl"))
        groups.append(("worker_cpu", ranks, "gloo"))
    for d in range(sae_dp_size):
        groups.append(("sae_tp", list(range(d * rep, d * rep + sae_tp_size)), "nccl"))
    for d in range(sae_dp_size):
        groups.append(("vllm_tp", list(range(d * rep, d * rep + vllm_tp_size)), "nccl"))
    for t in range(sae_tp_size):
        groups.append(("sae_dp", [d * rep + t for d in range(sae_dp_size)], "nccl"))
    return PrefixLayout("matched_dp" if matched else "local_overlap", world_size, sae_tp_size, sae_dp_size,
                        vllm_tp_size, sae_dp_size if matched else 1, rep, rep, groups, roles)


@dataclass
class RoutedLayout:
    """Layout of `init_distributed_v2` (P producers x Q consumers)."""

    P: int
    Q: int
    vllm_tp_size: int
    sae_tp_size: int
    disjoint: bool
    world_size: int
    producer_ranks: dict[int, list[int]]
    consumer_ranks: dict[int, list[int]]
    routing_table: list[ShardRoute]
    groups: list[tuple[str, list[int], str, int]]  # (kind, ranks, backend, index)

    @property
    def producer_tp_root(self) -> dict[int, int]:
        return {p: r[0] for p, r in self.producer_ranks.items()}

    @property
    def consumer_tp_root(self) -> dict[int, int]:
        return {c: r[0] for c, r in self.consumer_ranks.items()}

    def roles_of(self, rank: int) -> dict[str, int | bool]:
        out: dict[str, int | bool] = {"is_producer": False, "is_consumer": False, "producer_idx": -1,
                                      "consumer_idx": -1, "vllm_tp_rank": -1, "sae_tp_rank": -1}
        for p, ranks in self.producer_ranks.items():
            if rank in ranks:
                out.update(is_producer=True, producer_idx=p, vllm_tp_rank=ranks.index(rank))
        for c, ranks in self.consumer_ranks.items():
            if rank in ranks:
                out.update(is_consumer=True, consumer_idx=c, sae_tp_rank=ranks.index(rank))
        return out


def routed_layout(P: int, Q: int, vllm_tp_size: int, sae_tp_size: int, batch_size: int,
                  disjoint: bool = False) -> RoutedLayout:
    world = P * vllm_tp_size + Q * sae_tp_size if disjoint else max(P * vllm_tp_size, Q * sae_tp_size)
    prod = {p: list(range(p * vllm_tp_size, (p + 1) * vllm_tp_size)) for p in range(P)}
    off = P * vllm_tp_size if disjoint else 0
    cons = {c: list(range(off + c * sae_tp_size, off + (c + 1) * sae_tp_size)) for c in range(Q)}
    table = compute_routing_table(P, Q, batch_size) if P > 0 and Q > 0 else []
    groups: list[tuple[str, list[int], str, int]] = []
    for p in range(P):
        groups.append(("vllm_tp", prod[p], "nccl", p))
    for c in range(Q):
        groups.append(("sae_tp", cons[c], "nccl", c))
    for t in range(sae_tp_size):
        groups.append(("sae_dp", [cons[c][t] for c in range(Q)], "nccl", t))
    for c in range(Q):
        sources = {r.producer_idx for r in table if r.consumer_idx == c}
        members = sorted({cons[c][0]} | {prod[p][0] for p in sources})
        groups.append(("consumer_p2p", members, "nccl", c))
    return RoutedLayout(P, Q, vllm_tp_size, sae_tp_size, disjoint, world, prod, cons, table, groups)
