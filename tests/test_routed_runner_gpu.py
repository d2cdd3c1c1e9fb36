"""Shard-routing mode on 2 GPUs with the P2P row router: a disjoint producer -> consumer pair
(TopK on the native engine) and two co-located producer+consumer ranks (native DDP engine)."""

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


def _worker(rank, world, port, tmp, P, Q):
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
        save_mse_every_n_steps=1, n_checkpoints=0, verbose=False, sae_dp_mode="ddp" if Q > 1 else "manual")
    runner = LanguageModelSAETrainingRunner(cfg, override_model=lm, vllm_dp_size=P, sae_dp_size=Q,
                                            use_shard_routing=True)
    out = runner.run()
    info = {"role": runner.role, "transport": runner.routing_transport}
    if out is not None:
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
