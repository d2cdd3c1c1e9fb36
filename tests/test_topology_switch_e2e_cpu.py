"""End-to-end topology switch on CPU: the supervisor launches a streaming worker group through
torchrun (gloo, LM producer + SAE consumer, /dev/shm-style ring in a temp dir), a switch request
arrives mid-run, both roles quiesce (dataset position, SAE checkpoint, acks), the supervisor
restarts the group from the quiesce checkpoint and the run completes."""

import json
import os
import socket
import subprocess
import threading
import time
from pathlib import Path

import pytest

from saelens_b200.runners.topology_supervisor import (
    TopologySupervisor,
    build_torchrun_cmd,
    request_topology_switch,
)
from saelens_b200.topology_control import BufferParams, TopologySpec

REPO = Path(__file__).resolve().parents[1]


def _port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


@pytest.mark.timeout(400)
def test_topology_switch_quiesce_restart_complete(tmp_path):
    run_dir = tmp_path / "run"
    ring_dir = tmp_path / "ring"
    ring_dir.mkdir()
    out = run_dir / "out"
    steps, batch, chunk = 400, 64, 256
    worker_cfg = [
        "--architecture", "topk", "--d_in", "64", "--d_sae", "128", "--k", "8", "--model_name", "gpt2",
        "--model_from_pretrained_kwargs",
        json.dumps({"n_layers": 2, "d_model": 64, "n_heads": 4, "d_mlp": 128, "d_vocab": 500, "n_ctx": 64}),
        "--hook_name", "blocks.1.hook_resid_pre", "--dataset_path", "synthetic:uniform:500:32",
        "--context_size", "16", "--training_tokens", str(steps * batch), "--train_batch_size_tokens", str(batch),
        "--store_batch_size_prompts", "4", "--n_batches_in_buffer", "2", "--device", "cpu", "--output_path", str(out),
        "--streaming_chunk_size_tokens", str(chunk), "--streaming_num_chunks", "4", "--streaming_prefetch_chunks",
        "1", "--streaming_buffer_dir", str(ring_dir), "--save_mse_every_n_steps", "1", "--n_checkpoints", "0",
        "--log_to_wandb", "false", "--verbose", "false",
    ]
    env = dict(os.environ, PYTHONPATH=str(REPO) + os.pathsep + os.environ.get("PYTHONPATH", ""),
               OMP_NUM_THREADS="1")

    def launch(state):
        cmd = build_torchrun_cmd("-m saelens_b200.runners.worker", state.topology, run_dir, worker_cfg, port=_port())
        if state.checkpoint_path:
            cmd += ["--resume-from-checkpoint", state.checkpoint_path]
        log = open(run_dir / f"workers_{state.epoch}.log", "w")
        return subprocess.Popen(cmd, env=env, cwd=str(REPO), stdout=log, stderr=subprocess.STDOUT,
                                start_new_session=True)

    sup = TopologySupervisor(run_dir, TopologySpec(1, 1, 1, 1), launch, buffer_name=f"ring_{_port()}",
                             buffer_params=BufferParams(4, chunk, 64, "float32"), target_chunks=steps * batch // chunk,
                             buffer_base_dir=str(ring_dir), poll_s=0.3, exit_timeout_s=60.0, ack_timeout_s=120.0)
    result = {}
    th = threading.Thread(target=lambda: result.setdefault("rc", sup.run()), daemon=True)
    th.start()
    mse = out / "mse_history.jsonl"
    t0 = time.time()
    while not (mse.exists() and len(mse.read_text().splitlines()) >= 40):
        assert th.is_alive(), (run_dir / "workers_0.log").read_text()[-3000:]
        assert time.time() - t0 < 240, "no training progress"
        time.sleep(0.2)
    request_topology_switch(run_dir, TopologySpec(1, 1, 1, 1))
    th.join(timeout=300)
    assert not th.is_alive(), "supervisor did not finish"
    logs = "\n".join(p.read_text()[-2000:] for p in sorted(run_dir.glob("workers_*.log")))
    assert result.get("rc") == 0, logs
    events = [json.loads(x)["event"] for x in (run_dir / "topology_switch_log.jsonl").read_text().splitlines()]
    for e in ("switch_triggered", "quiesce_signaled", "all_acks_received", "checkpoint_found", "run_complete"):
        assert e in events, (events, logs)
    assert list((run_dir / "checkpoints").rglob("quiesce_*")), logs
    assert (run_dir / "producer_dataset_state_0").exists()
    assert (out / "sae_weights.safetensors").exists(), logs
