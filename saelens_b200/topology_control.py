"""Crash-consistent control state shared by the topology supervisor and its workers.

The supervisor rewrites `control_state.json` (write to a temporary file, then rename) before
every transition; workers read it at start-up to learn their topology, the activation ring and
the checkpoint to resume from (role of sae_lens/topology_control.py).
"""

from __future__ import annotations

import json
import os
from dataclasses import asdict, dataclass
from pathlib import Path

PHASES = ("RUNNING", "QUIESCING", "RESTARTING", "DONE")


@dataclass
class TopologySpec:
    vllm_tp: int
    vllm_dp: int
    sae_tp: int
    sae_dp: int = 1  # 0: producers only

    @property
    def world_size(self) -> int:
        return self.vllm_tp * self.vllm_dp + self.sae_tp * self.sae_dp


@dataclass
class BufferParams:
    num_chunks: int
    chunk_size_tokens: int
    d_model: int
    dtype: str  # "bfloat16" | "float32"
    num_hooks: int = 1


@dataclass
class ControlState:
    phase: str
    topology: TopologySpec
    buffer_name: str
    buffer_params: BufferParams
    checkpoint_path: str | None
    next_claim_seq_at_quiesce: int
    target_chunks: int
    epoch: int = 0

    def __post_init__(self) -> None:
        if self.phase not in PHASES:
            raise ValueError(f"phase must be one of {PHASES}, got {self.phase!r}")


def write_control_state(path: Path | str, state: ControlState) -> None:
    path = Path(path)
    path.parent.mkdir(parents=True, exist_ok=True)
    tmp = path.with_name(path.name + f".tmp{os.getpid()}")
    payload = asdict(state)
    with open(tmp, "w") as f:
        json.dump(payload, f, indent=2)
        f.flush()
        os.fsync(f.fileno())
    os.replace(tmp, path)


def read_control_state(path: Path | str) -> ControlState:
    d = json.loads(Path(path).read_text())
    topo = dict(d["topology"])
    topo.setdefault("sae_dp", 1)
    return ControlState(phase=d["phase"], topology=TopologySpec(**topo), buffer_name=d["buffer_name"],
                        buffer_params=BufferParams(**d["buffer_params"]), checkpoint_path=d.get("checkpoint_path"),
                        next_claim_seq_at_quiesce=d["next_claim_seq_at_quiesce"], target_chunks=d["target_chunks"],
                        epoch=d.get("epoch", 0))
