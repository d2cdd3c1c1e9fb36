"""torchrun worker entry and the supervisor's worker command."""

import sys

from saelens_b200.runners.topology_supervisor import build_torchrun_cmd
from saelens_b200.runners.worker import parse
from saelens_b200.topology_control import BufferParams, ControlState, TopologySpec, write_control_state

_CFG = ["--architecture", "topk", "--d_in", "64", "--d_sae", "128", "--k", "8", "--model_name", "gpt2",
        "--hook_name", "blocks.1.hook_resid_pre", "--dataset_path", "synthetic:uniform:500:32", "--device", "cpu"]


def test_worker_flags_and_config_fields():
    known, cfg = parse(["--vllm-dp-size", "2", "--sae-dp-size", "3", "--use-shard-routing", *_CFG])
    assert (known.vllm_dp_size, known.sae_dp_size, known.use_shard_routing) == (2, 3, True)
    assert cfg.sae.k == 8 and cfg.sae.d_sae == 128 and cfg.hook_name == "blocks.1.hook_resid_pre"
    assert known.run_dir is None and known.resume_from_checkpoint is None


def test_worker_under_supervisor_reads_control_state(tmp_path):
    write_control_state(tmp_path / "control_state.json", ControlState(
        phase="RUNNING", topology=TopologySpec(1, 1, 1, 1), buffer_name="ring_x",
        buffer_params=BufferParams(8, 128, 1, "bfloat16"), checkpoint_path=str(tmp_path / "ck" / "quiesce_64"),
        next_claim_seq_at_quiesce=0, target_chunks=10))
    known, cfg = parse(["--run-dir", str(tmp_path), "--streaming-mode", *_CFG])
    assert known.streaming_mode
    assert cfg.streaming_buffer_name == "ring_x" and cfg.streaming_transport == "host"
    assert cfg.checkpoint_path == str(tmp_path / "checkpoints")
    assert known.resume_from_checkpoint == str(tmp_path / "ck" / "quiesce_64")


def test_supervisor_launches_worker_module_with_topology(tmp_path):
    cmd = build_torchrun_cmd("-m saelens_b200.runners.worker", TopologySpec(1, 2, 2, 1), tmp_path, ["--k", "8"],
                             port=1234)
    assert cmd[:3] == [sys.executable, "-m", "torch.distributed.run"]
    i = cmd.index("-m", 3)
    assert cmd[i + 1] == "saelens_b200.runners.worker"
    for flag in ("--vllm-tp-size=1", "--vllm-dp-size=2", "--sae-tp-size=2", "--sae-dp-size=1", "--streaming-mode"):
        assert flag in cmd
    assert "--nproc-per-node=4" in cmd and cmd[-2:] == ["--k", "8"]


def test_supervisor_main_derives_ring_geometry_from_worker_args(tmp_path, monkeypatch):
    import saelens_b200.runners.topology_supervisor as ts

    seen = {}

    class FakeSup:
        def __init__(self, run_dir, topo, launch, **kw):
            seen.update(kw, topo=topo)

        def run(self):
            return 0

    monkeypatch.setattr(ts, "TopologySupervisor", FakeSup)
    rc = ts.main(["--run-dir", str(tmp_path), "--num-gpus", "2", "--buffer-base-dir", str(tmp_path),
                  *_CFG, "--streaming_num_chunks", "8", "--streaming_chunk_size_tokens", "512",
                  "--training_tokens", "5000"])
    assert rc == 0
    bp = seen["buffer_params"]
    assert (bp.num_chunks, bp.chunk_size_tokens, bp.d_model) == (8, 512, 64)
    assert seen["target_chunks"] == 10 and seen["buffer_base_dir"] == str(tmp_path)
