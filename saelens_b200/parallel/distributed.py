"""Process groups for the prefix-overlap topologies (local overlap, matched DP, fan-in).

API of sae_lens/distributed.py (init_distributed + getters + tp_allgather / tp_allreduce); the
rank arithmetic lives in `saelens_b200.parallel.layout.prefix_layout`.  Every rank creates every
group in the layout's order, as `torch.distributed.new_group` requires.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import torch.distributed as dist

from saelens_b200.parallel.layout import PrefixLayout, prefix_layout
from saelens_b200.parallel.tp import tp_allgather, tp_allreduce  # noqa: F401  (re-export)


@dataclass
class _State:
    layout: PrefixLayout | None = None
    rank: int = 0
    groups: dict[str, object] = field(default_factory=dict)


_S = _State()


def _reset() -> None:
    global _S
    _S = _State()


def init_distributed(tp_size: int | None = None, sae_dp_size: int = 1, *, sae_tp_size: int | None = None,
                     vllm_tp_size: int = 1, vllm_dp_size: int = 1, shared_tp_size: int | None = None) -> None:
    """Create the producer/trainer groups after `dist.init_process_group()`.

    `tp_size` (legacy) / `shared_tp_size` set one TP size for both the LM and the SAE.
    """
    if shared_tp_size is None and tp_size is not None and sae_tp_size is None:
        shared_tp_size = tp_size
    if shared_tp_size is not None:
        if vllm_dp_size > 1:
            raise ValueError("shared_tp_size is incompatible with vllm_dp_size > 1")
        if sae_tp_size is not None and sae_tp_size != shared_tp_size:
            raise ValueError(f"shared_tp_size={shared_tp_size} conflicts with sae_tp_size={sae_tp_size}")
        if vllm_tp_size not in (1, shared_tp_size):
            raise ValueError(f"shared_tp_size={shared_tp_size} conflicts with vllm_tp_size={vllm_tp_size}")
        sae_tp_size = vllm_tp_size = shared_tp_size
    if not dist.is_initialized():
        raise RuntimeError("Call dist.init_process_group() before init_distributed()")
    lay = prefix_layout(dist.get_world_size(), sae_tp_size or 1, sae_dp_size, vllm_tp_size, vllm_dp_size)
    rank = dist.get_rank()
    groups: dict[str, object] = {}
    for kind, ranks, backend in lay.groups:
        g = dist.new_group(ranks, backend=backend if backend == "gloo" else None)
        if rank not in ranks:
            continue
        role = lay.role(rank)
        if kind == "sae_tp" and not role.sae_active:
            continue
        if kind == "vllm_tp" and not role.vllm_active:
            continue
        if kind == "worker_cpu":
            groups["worker_cpu"] = g
            if lay.mode == "vllm_dp_fan_in":
                groups.setdefault("worker", groups.get("vllm_tp"))
            continue
        groups[kind] = g
        if lay.mode == "vllm_dp_fan_in" and kind == "vllm_tp":
            groups["worker"] = g
    _S.layout, _S.rank, _S.groups = lay, rank, groups


def _role():
    return None if _S.layout is None else _S.layout.role(_S.rank)


def is_distributed() -> bool:
    return dist.is_available() and dist.is_initialized() and dist.get_world_size() > 1


def get_worker_group():
    return _S.groups.get("worker")


def get_worker_cpu_group():
    return _S.groups.get("worker_cpu")


def get_worker_rank() -> int:
    r = _role()
    return 0 if r is None else r.worker_rank


def get_worker_size() -> int:
    return 1 if _S.layout is None else _S.layout.worker_size


def is_worker_active() -> bool:
    r = _role()
    return True if r is None else (r.vllm_active or r.sae_active)


def is_sae_active() -> bool:
    r = _role()
    return True if r is None else r.sae_active


def is_vllm_active() -> bool:
    r = _role()
    return True if r is None else r.vllm_active


def get_replica_base_rank() -> int:
    if _S.layout is None:
        return 0
    return (_S.rank // _S.layout.cluster_block) * _S.layout.cluster_block


def get_vllm_world_ranks() -> list[int]:
    """World ranks of this rank's LM TP group."""
    if _S.layout is None:
        return [0]
    ranks = _S.layout.group_of("vllm_tp", _S.rank)
    return ranks if ranks is not None else []


def get_vllm_root_rank() -> int:
    ranks = get_vllm_world_ranks()
    return ranks[0] if ranks else -1


def get_sae_root_rank() -> int:
    return get_replica_base_rank()


def get_sae_tp_group():
    return _S.groups.get("sae_tp")


get_tp_group = get_sae_tp_group


def get_sae_dp_group():
    return _S.groups.get("sae_dp")


get_dp_group = get_sae_dp_group


def get_vllm_tp_group():
    return _S.groups.get("vllm_tp")


def get_vllm_dp_p2p_group():
    return _S.groups.get("vllm_dp_p2p")


def get_sae_tp_rank() -> int:
    r = _role()
    return 0 if r is None else r.sae_tp_rank


get_tp_rank = get_sae_tp_rank


def get_sae_tp_size() -> int:
    return 1 if _S.layout is None else _S.layout.sae_tp_size


get_tp_size = get_sae_tp_size


def get_sae_dp_rank() -> int:
    r = _role()
    return 0 if r is None else r.sae_dp_rank


get_dp_rank = get_sae_dp_rank


def get_sae_dp_size() -> int:
    return 1 if _S.layout is None else _S.layout.sae_dp_size


get_dp_size = get_sae_dp_size


def get_vllm_tp_rank() -> int:
    r = _role()
    return 0 if r is None else r.vllm_tp_rank


def get_vllm_tp_size() -> int:
    return 1 if _S.layout is None else _S.layout.vllm_tp_size


def get_vllm_dp_rank() -> int:
    r = _role()
    return 0 if r is None else r.vllm_dp_rank


def get_vllm_dp_size() -> int:
    return 1 if _S.layout is None else _S.layout.vllm_dp_size


def is_vllm_dp_root() -> bool:
    return get_vllm_tp_rank() == 0


def get_layout_mode() -> str:
    return "local_overlap" if _S.layout is None else _S.layout.mode


def get_cluster_block() -> int:
    return 1 if _S.layout is None else _S.layout.cluster_block


def preinit_vllm_distributed(*_args, **_kwargs) -> None:
    """The reference pre-creates a vLLM fork's parallel state here.  The producer LMs of this
    package use the groups created by `init_distributed` directly, so nothing is needed."""
    return None
