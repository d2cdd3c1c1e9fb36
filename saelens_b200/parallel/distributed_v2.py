"""Process groups for P producer x Q consumer shard routing (API of sae_lens/distributed_v2.py)."""

from __future__ import annotations

from dataclasses import dataclass, field

import torch.distributed as dist

from saelens_b200.parallel.layout import RoutedLayout, routed_layout
from saelens_b200.parallel.shard_routing import ShardRoute


@dataclass
class _State:
    layout: RoutedLayout | None = None
    rank: int = 0
    groups: dict[str, object] = field(default_factory=dict)
    p2p: dict[int, object] = field(default_factory=dict)


_S = _State()
_initialized = False


def _reset() -> None:
    global _S, _initialized
    _S = _State()
    _initialized = False


def init_distributed_v2(P: int, Q: int, vllm_tp_size: int, sae_tp_size: int, batch_size: int,
                        disjoint: bool = False) -> None:
    global _initialized
    if not dist.is_initialized():
        raise RuntimeError("Call dist.init_process_group() before init_distributed_v2()")
    lay = routed_layout(P, Q, vllm_tp_size, sae_tp_size, batch_size, disjoint)
    if dist.get_world_size() != lay.world_size:
        raise ValueError(
            f"world_size={dist.get_world_size()} != {lay.world_size} for P={P}, vllm_tp={vllm_tp_size}, Q={Q}, "
            f"sae_tp={sae_tp_size}, disjoint={disjoint}"
        )
    rank = dist.get_rank()
    roles = lay.roles_of(rank)
    groups: dict[str, object] = {}
    p2p: dict[int, object] = {}
    on_nccl = dist.get_backend() == "nccl"
    for kind, ranks, backend, i in lay.groups:
        # device groups are NCCL on GPUs; a CPU (gloo) world uses its own backend for them
        g = dist.new_group(ranks, backend=backend if (on_nccl or backend != "nccl") else None)
        if rank not in ranks:
            continue
        if kind == "vllm_tp" and roles["producer_idx"] == i:
            groups["vllm_tp"] = g
        elif kind == "sae_tp" and roles["consumer_idx"] == i:
            groups["sae_tp"] = g
        elif kind == "sae_dp" and roles["sae_tp_rank"] == i:
            groups["sae_dp"] = g
        elif kind == "consumer_p2p":
            p2p[i] = g
    _S.layout, _S.rank, _S.groups, _S.p2p = lay, rank, groups, p2p
    _initialized = True


def _roles() -> dict:
    if _S.layout is None:
        return {"is_producer": False, "is_consumer": False, "producer_idx": -1, "consumer_idx": -1,
                "vllm_tp_rank": -1, "sae_tp_rank": -1}
    return _S.layout.roles_of(_S.rank)


def is_initialized() -> bool:
    return _initialized


def is_producer() -> bool:
    return bool(_roles()["is_producer"])


def is_consumer() -> bool:
    return bool(_roles()["is_consumer"])


def get_producer_idx() -> int:
    return int(_roles()["producer_idx"])


def get_consumer_idx() -> int:
    return int(_roles()["consumer_idx"])


def get_vllm_tp_rank() -> int:
    return int(_roles()["vllm_tp_rank"])


def get_sae_tp_rank() -> int:
    return int(_roles()["sae_tp_rank"])


def get_vllm_tp_size() -> int:
    return 0 if _S.layout is None else _S.layout.vllm_tp_size


def get_sae_tp_size() -> int:
    return 0 if _S.layout is None else _S.layout.sae_tp_size


def get_sae_dp_size() -> int:
    return 0 if _S.layout is None else _S.layout.Q


def get_routing_table() -> list[ShardRoute]:
    return [] if _S.layout is None else list(_S.layout.routing_table)


def get_vllm_tp_group():
    return _S.groups.get("vllm_tp")


def get_sae_tp_group():
    return _S.groups.get("sae_tp")


def get_sae_dp_group():
    return _S.groups.get("sae_dp")


def get_p2p_group(consumer_idx: int):
    return _S.p2p.get(consumer_idx)


def get_producer_tp_root(p: int) -> int:
    assert _S.layout is not None
    return _S.layout.producer_tp_root[p]


def get_consumer_tp_root(c: int) -> int:
    assert _S.layout is not None
    return _S.layout.consumer_tp_root[c]


def get_layout() -> RoutedLayout | None:
    return _S.layout
