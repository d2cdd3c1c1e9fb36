"""torchrun worker entry of the LM training runner (role of the reference's
scripts/run_sae_runner_gpu.py): distributed sizes and modes come from flags, every other
`--field value` is a config field (see `llm_sae_training_runner._parse_cfg_args`).

    python -m torch.distributed.run --nproc-per-node 8 --master-addr 127.0.0.1 \\
        -m saelens_b200.runners.worker --vllm-dp-size 2 --sae-dp-size 6 --use-shard-routing \\
        --architecture topk --d_in 4096 --d_sae 131072 --k 64 ...

Under the topology supervisor (`--run-dir`), the run directory holds the control state (ring name
and quota), the quiesce request and the acks; checkpoints go to `<run-dir>/checkpoints` unless
`--checkpoint_path` says otherwise, and the /dev/shm ring keeps READY chunks across restarts.
"""

from __future__ import annotations

import argparse
import sys
from pathlib import Path
from typing import Any


def parse(argv: list[str]) -> tuple[argparse.Namespace, Any]:
    from saelens_b200.runners.llm_sae_training_runner import _parse_cfg_args

    ap = argparse.ArgumentParser(prog="python -m saelens_b200.runners.worker", add_help=True)
    ap.add_argument("--run-dir", default=None)
    ap.add_argument("--vllm-tp-size", type=int, default=1)
    ap.add_argument("--vllm-dp-size", type=int, default=1)
    ap.add_argument("--sae-tp-size", type=int, default=1)
    ap.add_argument("--sae-dp-size", type=int, default=1)
    ap.add_argument("--streaming-mode", action="store_true")
    ap.add_argument("--use-shard-routing", action="store_true")
    ap.add_argument("--resume-from-checkpoint", default=None)
    known, rest = ap.parse_known_args(argv)
    cfg = _parse_cfg_args(rest)
    if known.run_dir is not None:
        run_dir = Path(known.run_dir)
        if not any(a.split("=")[0] in ("--checkpoint_path", "--checkpoint-path") for a in rest):
            cfg.checkpoint_path = str(run_dir / "checkpoints")  # where the supervisor looks for quiesce_*
        ctl = run_dir / "control_state.json"
        if ctl.exists():
            from saelens_b200.topology_control import read_control_state

            state = read_control_state(ctl)
            cfg.streaming_buffer_name = state.buffer_name
            if cfg.streaming_transport == "auto":
                cfg.streaming_transport = "host"  # READY chunks must outlive a topology switch
            if known.resume_from_checkpoint is None and state.checkpoint_path:
                known.resume_from_checkpoint = state.checkpoint_path
    return known, cfg


def main(argv: list[str] | None = None) -> Any:
    from saelens_b200.runners.llm_sae_training_runner import LanguageModelSAETrainingRunner

    known, cfg = parse(sys.argv[1:] if argv is None else argv)
    runner = LanguageModelSAETrainingRunner(
        cfg, resume_from_checkpoint=known.resume_from_checkpoint, sae_tp_size=known.sae_tp_size,
        sae_dp_size=known.sae_dp_size, vllm_tp_size=known.vllm_tp_size, vllm_dp_size=known.vllm_dp_size,
        use_shard_routing=known.use_shard_routing, streaming_mode=True if known.streaming_mode else None)
    if known.run_dir is not None:
        runner.quiesce_dir = known.run_dir
    out = runner.run()
    import torch.distributed as dist

    if dist.is_available() and dist.is_initialized():  # every rank leaves together
        dist.barrier()
        dist.destroy_process_group()
    return out


if __name__ == "__main__":
    main()
