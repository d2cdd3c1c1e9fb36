"""Shared activation ring, streaming provider, control state and the topology supervisor.

Faults are injected on the host only: worker processes that exit non-zero, hang through a
quiesce, or never acknowledge it; no GPU is involved."""

import json
import multiprocessing as mp
import os
import subprocess
import sys
import textwrap
import time

import pytest
import torch

from saelens_b200.runners.topology_supervisor import (
    TopologySupervisor,
    find_latest_quiesce_checkpoint,
    request_topology_switch,
)
from saelens_b200.topology_control import BufferParams, ControlState, TopologySpec, read_control_state, write_control_state
from saelens_b200.training.shared_activation_buffer import ChunkState, SharedActivationBuffer
from saelens_b200.training.streaming_activation_provider import StreamingActivationProvider


def _buf(tmp_path, create=True, **kw):
    args = dict(name="ring", num_chunks=4, chunk_size_tokens=8, d_model=4, num_producers=1, target_chunks=10,
                base_dir=str(tmp_path))
    args.update(kw)
    return SharedActivationBuffer(create=create, **args)


def test_ring_state_machine_and_roundtrip(tmp_path):
    b = _buf(tmp_path)
    slot, seq = b.allocate_write_chunk()
    assert seq == 0 and b.queue_counts()["writing"] == 1
    x = torch.randn(8, 4).to(torch.bfloat16)
    b.write_chunk(slot, x, valid_tokens=6)
    b.mark_ready(slot)
    idx, _ = b.acquire_up_to(4)
    assert idx == [slot]
    got, n = b.read_chunk(slot)
    assert n == 6 and torch.equal(got, x[:6])
    b.release_chunk(slot)
    assert b.queue_counts() == {"free": 4, "writing": 0, "ready": 0, "consuming": 0}
    with pytest.raises(RuntimeError):
        b.release_chunk(slot)
    b.signal_done()
    with pytest.raises(StopIteration):
        b.acquire_up_to(1)


def test_ring_quota_and_attach(tmp_path):
    b = _buf(tmp_path, target_chunks=2)
    assert b.allocate_write_chunk() is not None and b.allocate_write_chunk() is not None
    assert b.allocate_write_chunk() is None  # global quota used
    other = _buf(tmp_path, create=False)
    assert other.next_claim_seq == 2
    assert other.queue_counts()["writing"] == 2


def test_reset_for_restart_recycles_writing_slots(tmp_path):
    b = _buf(tmp_path, num_producers=2)
    s, _ = b.allocate_write_chunk()
    b.signal_done()
    b.reset_for_restart(3)
    assert b.queue_counts()["free"] == 4 and b.num_producers == 3 and b.done_count == 0
    assert int(b._slots[s, 0]) == ChunkState.FREE


def _producer_proc(base, name, pid_, n_rows):
    b = SharedActivationBuffer(name, 4, 8, 4, num_producers=2, base_dir=base)
    while True:
        got = b.allocate_write_chunk()
        if got is None:
            break
        s, seq = got
        b.write_chunk(s, torch.full((8, 4), float(seq)), valid_tokens=8, producer_id=pid_)
        b.mark_ready(s)
    b.signal_done()


def test_two_producer_processes_one_consumer(tmp_path):
    b = SharedActivationBuffer("mp", 4, 8, 4, num_producers=2, target_chunks=12, create=True,
                               base_dir=str(tmp_path), dtype=torch.float32)
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_producer_proc, args=(str(tmp_path), "mp", i, 8)) for i in range(2)]
    for p in procs:
        p.start()
    prov = StreamingActivationProvider(b, train_batch_size_tokens=16, prefetch_chunks=2, device="cpu", d_model=4,
                                       shuffle=False)
    seen = []
    for batch in prov:
        seen.append(batch)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    allrows = torch.cat(seen)
    assert allrows.shape[0] == 12 * 8  # every claimed chunk delivered exactly once
    assert sorted(set(allrows[:, 0].tolist())) == list(map(float, range(12)))


def test_provider_multi_hook_dicts(tmp_path):
    b = SharedActivationBuffer("mh", 4, 8, 2, num_producers=1, target_chunks=1, create=True,
                               base_dir=str(tmp_path), dtype=torch.float32)
    s, _ = b.allocate_write_chunk()
    rows = torch.cat([torch.zeros(4, 2), torch.ones(4, 2)])  # [hook0 block | hook1 block] of 4 tokens
    b.write_chunk(s, rows, 8)
    b.mark_ready(s)
    b.signal_done()
    prov = StreamingActivationProvider(b, train_batch_size_tokens=4, prefetch_chunks=1, device="cpu", d_model=2,
                                       hook_names=["a", "b"])
    out = next(prov)
    assert set(out) == {"a", "b"} and out["a"].shape == (4, 2)
    assert (out["a"] == 0).all() and (out["b"] == 1).all()


def test_control_state_atomic_roundtrip(tmp_path):
    st = ControlState("RUNNING", TopologySpec(2, 1, 1, 1), "buf", BufferParams(8, 16, 4, "bfloat16"), None, 0, 100)
    write_control_state(tmp_path / "c.json", st)
    back = read_control_state(tmp_path / "c.json")
    assert back == st and back.topology.world_size == 3
    assert not list(tmp_path.glob("*.tmp*"))
    with pytest.raises(ValueError):
        ControlState("BOGUS", st.topology, "b", st.buffer_params, None, 0, 0)


WORKER = textwrap.dedent("""
    import json, os, sys, time, pathlib
    run = pathlib.Path(sys.argv[1]); mode = sys.argv[2]
    st = json.loads((run / "control_state.json").read_text())
    (run / f"launch_{st['epoch']}").write_text(json.dumps(st["topology"]))
    if mode == "crash_once" and st["epoch"] == 0:
        sys.exit(3)
    for _ in range(400):
        if (run / "quiesce_request").exists():
            if mode == "ignore_quiesce":
                time.sleep(60)
            ck = run / "checkpoints" / "x" / f"quiesce_{100 + st['epoch']}"
            ck.mkdir(parents=True, exist_ok=True)
            for i in range(st["topology"]["vllm_dp"]):
                (run / f"quiesce_ack_producer_{i}").touch()
            (run / "quiesce_ack").touch()
            sys.exit(0)
        if mode == "finish" or (mode == "crash_once" and st["epoch"] >= 1) or (
                mode in ("switch", "ignore_quiesce") and st["epoch"] >= 1):
            sys.exit(0)
        time.sleep(0.05)
    sys.exit(0)
""")


def _sup(tmp_path, mode, **kw):
    script = tmp_path / "worker.py"
    script.write_text(WORKER)

    def launch(state):
        return subprocess.Popen([sys.executable, str(script), str(tmp_path), mode], start_new_session=True)

    return TopologySupervisor(tmp_path, TopologySpec(1, 2, 1, 1), launch, buffer_base_dir=str(tmp_path),
                              poll_s=0.05, exit_timeout_s=2.0, **kw)


def test_supervisor_restarts_crashed_workers(tmp_path):
    sup = _sup(tmp_path, "crash_once")
    assert sup.run() == 0
    assert sup.crash_restarts == 1
    assert (tmp_path / "launch_0").exists() and (tmp_path / "launch_1").exists()
    events = [json.loads(x)["event"] for x in (tmp_path / "topology_switch_log.jsonl").read_text().splitlines()]
    assert "workers_crashed" in events and events[-1] == "run_complete"


def test_supervisor_switches_topology_with_quiesce(tmp_path):
    sup = _sup(tmp_path, "switch")
    request_topology_switch(tmp_path, TopologySpec(1, 3, 1, 1))
    assert sup.run() == 0
    assert sup.switches == 1
    assert json.loads((tmp_path / "launch_1").read_text())["vllm_dp"] == 3
    st = read_control_state(tmp_path / "control_state.json")
    assert st.phase == "DONE" and st.checkpoint_path.endswith("quiesce_100")
    assert not (tmp_path / "quiesce_request").exists()


def test_supervisor_kills_workers_that_ignore_quiesce(tmp_path):
    sup = _sup(tmp_path, "ignore_quiesce", ack_timeout_s=0.5)
    request_topology_switch(tmp_path, TopologySpec(1, 1, 1, 1))
    t0 = time.time()
    assert sup.run() == 0
    assert time.time() - t0 < 30
    events = [json.loads(x)["event"] for x in (tmp_path / "topology_switch_log.jsonl").read_text().splitlines()]
    assert "ack_timeout" in events and "workers_killed" in events


def test_supervisor_gives_up_after_repeated_crashes(tmp_path):
    script = tmp_path / "bad.py"
    script.write_text("import sys; sys.exit(7)")
    sup = TopologySupervisor(tmp_path, TopologySpec(1, 1, 1, 1),
                             lambda st: subprocess.Popen([sys.executable, str(script)]), buffer_base_dir=str(tmp_path),
                             poll_s=0.05, max_crash_restarts=2)
    assert sup.run() == 7
    assert sup.crash_restarts == 2


def test_recovers_interrupted_switch(tmp_path):
    st = ControlState("QUIESCING", TopologySpec(1, 2, 1, 1), "buf", BufferParams(4, 8, 4, "bfloat16"), None, 0, 10)
    write_control_state(tmp_path / "control_state.json", st)
    (tmp_path / "checkpoints" / "r" / "quiesce_42").mkdir(parents=True)
    request_topology_switch(tmp_path, TopologySpec(1, 4, 1, 1))
    sup = TopologySupervisor(tmp_path, TopologySpec(1, 2, 1, 1), lambda s: None, buffer_base_dir=str(tmp_path))
    assert sup.state.topology.vllm_dp == 4
    assert sup.state.checkpoint_path.endswith("quiesce_42")
    assert find_latest_quiesce_checkpoint(tmp_path).endswith("quiesce_42")
