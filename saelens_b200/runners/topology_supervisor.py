"""Topology supervisor: runs streaming SAE training as a relaunchable worker group and switches
its producer/trainer topology mid-run (behaviour of scripts/topology_supervisor.py).

Loop (poll every `poll_s`):
* workers exited 0 and no switch pending -> done;
* workers crashed -> recycle abandoned ring slots, relaunch the same topology from the latest
  quiesce checkpoint (bounded by `max_crash_restarts`);
* `topology_request.json` appeared -> phase QUIESCING, touch `quiesce_request`; wait for one
  ack per producer (`quiesce_ack_producer_{i}`) and the trainer's `quiesce_ack`; wait for the
  workers to exit (kill them after `exit_timeout_s`); reset the ring for the new producer count;
  relaunch with the new topology, resuming from the newest `quiesce_*` checkpoint.

Everything here runs on the host: faults are injected by making workers exit, hang, or skip
their acks; no GPU is ever made to fault.
"""

from __future__ import annotations

import argparse
import json
import os
import signal
import socket
import subprocess
import sys
import time
from collections.abc import Callable
from dataclasses import asdict
from pathlib import Path
from typing import Any

from saelens_b200.topology_control import (
    BufferParams,
    ControlState,
    TopologySpec,
    read_control_state,
    write_control_state,
)

CONTROL_FILE = "control_state.json"
REQUEST_FILE = "topology_request.json"
QUIESCE_REQUEST = "quiesce_request"
CONSUMER_ACK = "quiesce_ack"
SWITCH_LOG = "topology_switch_log.jsonl"


class SwitchLog:
    def __init__(self, path: Path):
        self.path = path

    def write(self, event: str, **fields: Any) -> None:
        rec = {"event": event, "time": time.time(), **fields}
        with open(self.path, "a") as f:
            f.write(json.dumps(rec) + "\n")


def find_free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def build_torchrun_cmd(worker_script: str, topo: TopologySpec, run_dir: Path, extra_args: list[str],
                       port: int | None = None) -> list[str]:
    """torchrun command of one worker group; `worker_script` is a script path or `-m module`."""
    target = worker_script.split() if worker_script.startswith("-m ") else [worker_script]
    return [
        sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={topo.world_size}",
        "--master-addr", "127.0.0.1", f"--master-port={port or find_free_port()}", *target,
        "--run-dir", str(run_dir), "--streaming-mode", f"--vllm-tp-size={topo.vllm_tp}",
        f"--vllm-dp-size={topo.vllm_dp}", f"--sae-tp-size={topo.sae_tp}", f"--sae-dp-size={max(topo.sae_dp, 1)}",
        *extra_args,
    ]


def producer_ack_paths(run_dir: Path, vllm_dp: int) -> list[Path]:
    return [run_dir / f"quiesce_ack_producer_{i}" for i in range(vllm_dp)]


def all_acks_present(run_dir: Path, topo: TopologySpec) -> bool:
    acks = producer_ack_paths(run_dir, topo.vllm_dp)
    if topo.sae_dp > 0:
        acks.append(run_dir / CONSUMER_ACK)
    return all(p.exists() for p in acks)


def cleanup_quiesce_files(run_dir: Path, vllm_dp: int) -> None:
    for p in [run_dir / QUIESCE_REQUEST, run_dir / CONSUMER_ACK, *producer_ack_paths(run_dir, vllm_dp)]:
        p.unlink(missing_ok=True)


def find_latest_quiesce_checkpoint(run_dir: Path) -> str | None:
    """Newest `quiesce_<n>` directory (largest n) anywhere under run_dir/checkpoints."""
    best: tuple[int, str] | None = None
    root = run_dir / "checkpoints"
    if not root.exists():
        return None
    for p in root.rglob("quiesce_*"):
        if not p.is_dir():
            continue
        try:
            n = int(p.name.split("_", 1)[1])
        except ValueError:
            continue
        if best is None or n > best[0]:
            best = (n, str(p))
    return None if best is None else best[1]


def reset_buffer(state: ControlState, base_dir: str, new_num_producers: int) -> None:
    """Return abandoned WRITING slots to FREE and set the producer count (no worker alive)."""
    from saelens_b200.training.shared_activation_buffer import SharedActivationBuffer

    bp = state.buffer_params
    try:
        buf = SharedActivationBuffer(state.buffer_name, bp.num_chunks, bp.chunk_size_tokens * bp.num_hooks,
                                     bp.d_model, num_producers=new_num_producers, base_dir=base_dir)
    except FileNotFoundError:
        return
    buf.reset_for_restart(new_num_producers)
    buf.close()


class TopologySupervisor:
    def __init__(self, run_dir: str | Path, topology: TopologySpec, launch: Callable[[ControlState], subprocess.Popen],
                 buffer_name: str = "", buffer_params: BufferParams | None = None, target_chunks: int = 0,
                 buffer_base_dir: str = "/dev/shm", poll_s: float = 5.0, exit_timeout_s: float = 60.0,
                 ack_timeout_s: float = 600.0, max_crash_restarts: int = 3, resume_from_checkpoint: str | None = None):
        self.run_dir = Path(run_dir)
        self.run_dir.mkdir(parents=True, exist_ok=True)
        self.launch = launch
        self.poll_s = poll_s
        self.exit_timeout_s = exit_timeout_s
        self.ack_timeout_s = ack_timeout_s
        self.max_crash_restarts = max_crash_restarts
        self.base_dir = buffer_base_dir
        self.log = SwitchLog(self.run_dir / SWITCH_LOG)
        self.crash_restarts = 0
        self.switches = 0
        self.state = ControlState(
            phase="RUNNING", topology=topology, buffer_name=buffer_name or f"saeb_{os.getpid()}",
            buffer_params=buffer_params or BufferParams(32, 4096, 1, "bfloat16"),
            checkpoint_path=resume_from_checkpoint, next_claim_seq_at_quiesce=0, target_chunks=target_chunks,
        )
        self._recover_interrupted_quiesce()

    @property
    def control_path(self) -> Path:
        return self.run_dir / CONTROL_FILE

    def _recover_interrupted_quiesce(self) -> None:
        """A supervisor that died mid-switch left phase QUIESCING/RESTARTING: finish the switch
        from the last written state (the newest quiesce checkpoint and the requested topology)."""
        if not self.control_path.exists():
            return
        old = read_control_state(self.control_path)
        if old.phase in ("QUIESCING", "RESTARTING"):
            req = self.run_dir / REQUEST_FILE
            topo = old.topology
            if req.exists():
                topo = TopologySpec(**json.loads(req.read_text()))
                req.unlink()
            ck = find_latest_quiesce_checkpoint(self.run_dir) or old.checkpoint_path
            cleanup_quiesce_files(self.run_dir, old.topology.vllm_dp)
            self.state = ControlState("RUNNING", topo, old.buffer_name, old.buffer_params, ck,
                                      old.next_claim_seq_at_quiesce, old.target_chunks, old.epoch + 1)
            self.log.write("recovered_interrupted_switch", topology=asdict(topo), checkpoint=ck)

    def _write(self) -> None:
        write_control_state(self.control_path, self.state)

    def _start(self) -> subprocess.Popen:
        self._write()
        proc = self.launch(self.state)
        self.log.write("workers_launched", topology=asdict(self.state.topology), pid=proc.pid, epoch=self.state.epoch)
        return proc

    def _stop(self, proc: subprocess.Popen) -> int | None:
        t0 = time.time()
        while proc.poll() is None and time.time() - t0 < self.exit_timeout_s:
            time.sleep(min(self.poll_s, 0.2))
        if proc.poll() is None:
            try:
                os.killpg(proc.pid, signal.SIGKILL)
            except (ProcessLookupError, PermissionError, OSError):
                proc.kill()
            proc.wait()
            self.log.write("workers_killed", pid=proc.pid)
        return proc.returncode

    def run(self) -> int:
        self.log.write("supervisor_start", topology=asdict(self.state.topology), run_dir=str(self.run_dir))
        proc = self._start()
        while True:
            time.sleep(self.poll_s)
            req = self.run_dir / REQUEST_FILE
            rc = proc.poll()
            if rc is not None and not req.exists():
                if rc == 0:
                    self.state.phase = "DONE"
                    self._write()
                    self.log.write("run_complete", topology=asdict(self.state.topology))
                    return 0
                self.log.write("workers_crashed", exit_code=rc, topology=asdict(self.state.topology))
                if self.crash_restarts >= self.max_crash_restarts:
                    self.log.write("giving_up", crash_restarts=self.crash_restarts)
                    return rc
                self.crash_restarts += 1
                reset_buffer(self.state, self.base_dir, self.state.topology.vllm_dp)
                self.state.checkpoint_path = find_latest_quiesce_checkpoint(self.run_dir) or self.state.checkpoint_path
                self.state.epoch += 1
                proc = self._start()
                continue
            if req.exists():
                proc = self._switch(proc, req)

    def _switch(self, proc: subprocess.Popen, req: Path) -> subprocess.Popen:
        new_topo = TopologySpec(**json.loads(req.read_text()))
        old_topo = self.state.topology
        self.log.write("switch_triggered", from_topology=asdict(old_topo), to_topology=asdict(new_topo))
        self.state.phase = "QUIESCING"
        self._write()
        (self.run_dir / QUIESCE_REQUEST).touch()
        self.log.write("quiesce_signaled", from_topology=asdict(old_topo))
        t0 = time.time()
        while not all_acks_present(self.run_dir, old_topo) and proc.poll() is None:
            if time.time() - t0 > self.ack_timeout_s:
                self.log.write("ack_timeout", waited_s=time.time() - t0)
                break
            time.sleep(min(self.poll_s, 0.2))
        else:
            if all_acks_present(self.run_dir, old_topo):
                self.log.write("all_acks_received", from_topology=asdict(old_topo))
        rc = self._stop(proc)
        self.log.write("workers_exited", exit_code=rc, from_topology=asdict(old_topo))
        self.state.phase = "RESTARTING"
        self._write()
        ck = find_latest_quiesce_checkpoint(self.run_dir)
        self.log.write("checkpoint_found", checkpoint_path=ck)
        reset_buffer(self.state, self.base_dir, new_topo.vllm_dp)
        cleanup_quiesce_files(self.run_dir, old_topo.vllm_dp)
        req.unlink(missing_ok=True)
        self.state.topology = new_topo
        self.state.checkpoint_path = ck or self.state.checkpoint_path
        self.state.phase = "RUNNING"
        self.state.epoch += 1
        self.switches += 1
        return self._start()


def request_topology_switch(run_dir: str | Path, topology: TopologySpec) -> None:
    """What an operator (or a scheduler) does to trigger a switch."""
    p = Path(run_dir) / REQUEST_FILE
    tmp = p.with_name(p.name + ".tmp")
    tmp.write_text(json.dumps(asdict(topology)))
    os.replace(tmp, p)


def main(argv: list[str] | None = None) -> int:
    ap = argparse.ArgumentParser(description="Topology supervisor for streaming SAE training")
    ap.add_argument("--run-dir", required=True)
    ap.add_argument("--worker-script", default="-m saelens_b200.runners.worker")
    ap.add_argument("--vllm-tp", type=int, default=1)
    ap.add_argument("--vllm-dp", type=int, default=1)
    ap.add_argument("--sae-tp", type=int, default=1)
    ap.add_argument("--sae-dp", type=int, default=1)
    ap.add_argument("--num-gpus", type=int, required=True)
    ap.add_argument("--resume-from-checkpoint", default=None)
    ap.add_argument("--buffer-base-dir", default="/dev/shm")
    ap.add_argument("--poll-s", type=float, default=5.0)
    ap.add_argument("--exit-timeout-s", type=float, default=60.0)
    args, extra = ap.parse_known_args(argv)
    topo = TopologySpec(args.vllm_tp, args.vllm_dp, args.sae_tp, args.sae_dp)
    buffer_params, target_chunks = None, 0
    if extra:
        # the ring's geometry and quota come from the workers' own config fields
        import math

        from saelens_b200.runners.worker import parse as parse_worker

        extra = [*extra, "--streaming_buffer_dir", args.buffer_base_dir]
        _, wcfg = parse_worker(extra)
        n_hooks = len(wcfg.hook_names) if getattr(wcfg, "hook_names", None) else 1
        buffer_params = BufferParams(wcfg.streaming_num_chunks, wcfg.streaming_chunk_size_tokens, wcfg.sae.d_in,
                                     "float32" if wcfg.dtype in ("float32", "torch.float32") else "bfloat16",
                                     num_hooks=n_hooks)
        target_chunks = math.ceil(wcfg.training_tokens / wcfg.streaming_chunk_size_tokens)
    if topo.world_size > args.num_gpus:
        raise SystemExit(f"topology needs {topo.world_size} GPUs, only {args.num_gpus} available")
    run_dir = Path(args.run_dir)

    def launch(state: ControlState) -> subprocess.Popen:
        cmd = build_torchrun_cmd(args.worker_script, state.topology, run_dir, extra)
        if state.checkpoint_path:
            cmd += ["--resume-from-checkpoint", state.checkpoint_path]
        return subprocess.Popen(cmd, start_new_session=True)

    sup = TopologySupervisor(run_dir, topo, launch, buffer_params=buffer_params, target_chunks=target_chunks,
                             buffer_base_dir=args.buffer_base_dir, poll_s=args.poll_s,
                             exit_timeout_s=args.exit_timeout_s, resume_from_checkpoint=args.resume_from_checkpoint)
    return sup.run()


if __name__ == "__main__":
    raise SystemExit(main())
