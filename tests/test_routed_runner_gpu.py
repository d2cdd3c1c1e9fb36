"""Shard-routing mode on 2 GPUs with the P2P row router: a disjoint producer -> consumer pair
(TopK on the native engine), two co-located producer+consumer ranks (native DDP engine), one
producer feeding an SAE whose latents are sharded over both GPUs (the producer stores the rows
into each TP member's landing buffer), and two hooks routed side by side."""

import json
import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu


def _port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, tmp, P, Q, stp=1, hooks=None):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank), SAELENS_B200_ROUTE_WAIT_S="90")
    import torch.distributed as dist
    from datetime import timedelta

    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    from saelens_b200.config import LanguageModelSAERunnerConfig, LoggingConfig
    from saelens_b200.models.lm import HookedLM, preset_config
    from saelens_b200.models.topk import TopKTrainingSAEConfig
    from saelens_b200.runners.llm_sae_training_runner import LanguageModelSAETrainingRunner

    torch.manual_seed(0)
    lm = HookedLM(preset_config("gpt2", n_layers=2, d_model=128, n_heads=4, d_mlp=256, d_vocab=500, n_ctx=64,
                                dtype="float32")).to(f"cuda:{rank}")
    torch.manual_seed(1)
    cfg = LanguageModelSAERunnerConfig(
        sae=TopKTrainingSAEConfig(d_in=128, d_sae=512, k=8), model_name="gpt2", hook_name="blocks.1.hook_resid_pre",
        dataset_path="synthetic:uniform:500:32", context_size=16, training_tokens=256 * 8,
        train_batch_size_tokens=256, store_batch_size_prompts=8, n_batches_in_buffer=2,
        output_path=os.path.join(tmp, "out"), logger=LoggingConfig(log_to_wandb=False), device="cuda",
        save_mse_every_n_steps=1, n_checkpoints=0, verbose=False, sae_dp_mode="ddp" if Q > 1 else "manual",
        **({"hook_names": list(hooks)} if hooks else {}))
    runner = LanguageModelSAETrainingRunner(cfg, override_model=lm, vllm_dp_size=P, sae_dp_size=Q,
                                            sae_tp_size=stp, use_shard_routing=True)
    out = runner.run()
    info = {"role": runner.role, "transport": runner.routing_transport,
            "to_members": bool(getattr(runner, "route_to_members", False))}
    if isinstance(out, dict):
        info["steps"] = runner.trainer.n_training_steps
        info["W_dec_sum"] = {h: float(s.W_dec.detach().float().sum()) for h, s in out.items()}
    elif out is not None:
        info["steps"] = runner.trainer.n_training_steps
        info["engine"] = type(runner.trainer.engine).__name__
        info["W_dec_sum"] = float(out.W_dec.detach().float().sum())
    with open(os.path.join(tmp, f"r{rank}.json"), "w") as f:
        json.dump(info, f)
    dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("P,Q", [(1, 1), (2, 2)])
def test_routed_runner_p2p(tmp_path, P, Q):
    import torch.multiprocessing as mp

    mp.spawn(_worker, args=(2, _port(), str(tmp_path), P, Q), nprocs=2, join=True)
    r = [json.loads((tmp_path / f"r{i}.json").read_text()) for i in range(2)]
    if (P, Q) == (1, 1):
        assert r[0]["role"] == "producer" and r[1]["role"] == "consumer"
        assert r[1]["transport"] == "p2p" and r[1]["steps"] == 8 and r[1]["engine"] == "FusedTopKEngine"
    else:
        assert r[0]["role"] == r[1]["role"] == "producer+consumer"
        assert r[0]["engine"] == r[1]["engine"] == "DDPTopKEngine"
        assert r[0]["steps"] == r[1]["steps"] == 8 and r[0]["W_dec_sum"] == r[1]["W_dec_sum"]
    assert (tmp_path / "out" / "sae_weights.safetensors").exists()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_routed_runner_p2p_into_tensor_parallel_members(tmp_path):
    """P 1, Q 1 with SAE TP 2 on 2 GPUs: rank 0 produces and holds the first latent shard, rank 1
    the second; the router kernel stores every row into both members' landing buffers."""
    import torch.multiprocessing as mp

    mp.spawn(_worker, args=(2, _port(), str(tmp_path), 1, 1, 2), nprocs=2, join=True)
    r = [json.loads((tmp_path / f"r{i}.json").read_text()) for i in range(2)]
    assert r[0]["role"] == "producer+consumer" and r[1]["role"] == "consumer"
    assert r[0]["to_members"] and r[1]["to_members"]
    assert r[0]["steps"] == r[1]["steps"] == 8
    assert r[0]["engine"] == r[1]["engine"] == "TPTopKEngine"
    assert (tmp_path / "out" / "sae_weights.safetensors").exists()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_routed_runner_p2p_multi_hook(tmp_path):
    """Two hooks side by side in each routed row, two producer+consumer ranks (DDP replicas): one
    SAE per hook on each rank, equal across the replicas."""
    import torch.multiprocessing as mp

    hooks = ["blocks.0.hook_resid_pre", "blocks.1.hook_resid_pre"]
    mp.spawn(_worker, args=(2, _port(), str(tmp_path), 2, 2, 1, hooks), nprocs=2, join=True)
    r = [json.loads((tmp_path / f"r{i}.json").read_text()) for i in range(2)]
    assert r[0]["steps"] == r[1]["steps"] == 8
    for h in hooks:
        assert r[0]["W_dec_sum"][h] == pytest.approx(r[1]["W_dec_sum"][h], rel=1e-6)
    assert r[0]["W_dec_sum"][hooks[0]] != r[0]["W_dec_sum"][hooks[1]]
    subdirs = [p for p in (tmp_path / "out").iterdir() if p.is_dir()]
    assert len(subdirs) == 2
