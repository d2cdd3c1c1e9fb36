"""Legacy fan-in data path on CPU (gloo): helper producers serve activation batches to their
cluster's SAE root (m:1 with 2 producers, mn:m with 4 producers and 2 data-parallel roots)."""

import json
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp


def _port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, tmp, vdp, sdp):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    import torch.distributed as dist

    dist.init_process_group("gloo", rank=rank, world_size=world)
    from saelens_b200.config import LanguageModelSAERunnerConfig, LoggingConfig
    from saelens_b200.models.lm import HookedLM, preset_config
    from saelens_b200.models.standard import StandardTrainingSAEConfig
    from saelens_b200.runners import fan_in
    from saelens_b200.runners.llm_sae_training_runner import LanguageModelSAETrainingRunner

    sent = {}
    orig = fan_in.run_helper

    def counting(store, root, group):
        sent["n"] = orig(store, root, group)
        return sent["n"]

    fan_in.run_helper = counting
    torch.manual_seed(0)
    lm = HookedLM(preset_config("gpt2", n_layers=2, d_model=64, n_heads=4, d_mlp=128, d_vocab=500, n_ctx=64,
                                dtype="float32"))
    cfg = LanguageModelSAERunnerConfig(
        sae=StandardTrainingSAEConfig(d_in=64, d_sae=128, l1_coefficient=1e-3), model_name="gpt2",
        hook_name="blocks.1.hook_resid_pre", dataset_path="synthetic:uniform:500:32", context_size=16,
        training_tokens=64 * 6, train_batch_size_tokens=64, store_batch_size_prompts=4, n_batches_in_buffer=2,
        output_path=os.path.join(tmp, "out"), logger=LoggingConfig(log_to_wandb=False), device="cpu",
        n_checkpoints=0, verbose=False, sae_dp_mode="manual")
    runner = LanguageModelSAETrainingRunner(cfg, override_model=lm, vllm_dp_size=vdp, sae_dp_size=sdp)
    out = runner.run()
    info = {"role": runner.role, "fan_in": runner.fan_in, "sent": sent.get("n")}
    if out is not None:
        info["steps"] = runner.trainer.n_training_steps
        info["W_dec_sum"] = float(out.W_dec.detach().sum())
    with open(os.path.join(tmp, f"r{rank}.json"), "w") as f:
        json.dump(info, f)
    dist.destroy_process_group()


@pytest.mark.parametrize("world,vdp,sdp", [(2, 2, 1), (4, 4, 2)])
def test_fan_in_helpers_feed_sae_roots(tmp_path, world, vdp, sdp):
    mp.spawn(_worker, args=(world, _port(), str(tmp_path), vdp, sdp), nprocs=world, join=True)
    r = [json.loads((tmp_path / f"r{i}.json").read_text()) for i in range(world)]
    block = vdp // sdp
    for i, x in enumerate(r):
        assert x["fan_in"]
        if i % block == 0:
            assert x["role"] == "producer+consumer" and x["steps"] == 6
        else:
            assert x["role"] == "producer" and x["sent"] > 0
    if sdp > 1:  # data-parallel roots stay identical
        assert r[0]["W_dec_sum"] == pytest.approx(r[block]["W_dec_sum"], rel=1e-6)
    assert (tmp_path / "out" / "sae_weights.safetensors").exists()
