"""Disjoint producer / consumer GPU sets for streaming mode (API of
sae_lens/distributed_streaming.py): producers and trainers never share a rank and meet only in
the activation ring buffer.  At most one SAE DP replica: independent ring claims diverge at the
stream tail, which would desynchronise data-parallel collectives."""

from __future__ import annotations

from saelens_b200.parallel import distributed_v2 as _v2

_vllm_dp_size = 0


def init_distributed_streaming(vllm_tp: int, vllm_dp: int, sae_tp: int, sae_dp: int = 1) -> None:
    global _vllm_dp_size
    if sae_dp not in (0, 1):
        raise ValueError(
            f"streaming_mode v1 requires sae_dp in {{0, 1}}, got sae_dp={sae_dp}. sae_dp > 1 is not supported."
        )
    _vllm_dp_size = vllm_dp
    _v2.init_distributed_v2(P=vllm_dp, Q=sae_dp, vllm_tp_size=vllm_tp, sae_tp_size=sae_tp, batch_size=1,
                            disjoint=True)


is_producer = _v2.is_producer
is_consumer = _v2.is_consumer
get_producer_idx = _v2.get_producer_idx
get_vllm_tp_group = _v2.get_vllm_tp_group
get_sae_tp_group = _v2.get_sae_tp_group
get_sae_tp_rank = _v2.get_sae_tp_rank
get_sae_tp_size = _v2.get_sae_tp_size
get_vllm_tp_size = _v2.get_vllm_tp_size
get_vllm_tp_rank = _v2.get_vllm_tp_rank


def get_vllm_dp_size() -> int:
    return _vllm_dp_size


def get_producer_tp_root(p: int) -> int:
    return _v2.get_producer_tp_root(p)


def get_consumer_tp_root(c: int = 0) -> int:
    return _v2.get_consumer_tp_root(c)


def is_vllm_tp_root() -> bool:
    return _v2.is_producer() and _v2.get_vllm_tp_rank() == 0


def is_sae_tp_root() -> bool:
    return _v2.is_consumer() and _v2.get_sae_tp_rank() == 0
