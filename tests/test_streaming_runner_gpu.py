"""Streaming mode on 2 GPUs with the device ring: GPU 0 runs the LM and writes activation chunks
over NVLink into GPU 1's ring; GPU 1 trains a TopK SAE (native engine) from it."""

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


def _worker(rank, world, port, tmp):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
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
    cfg = LanguageModelSAERunnerConfig(
        sae=TopKTrainingSAEConfig(d_in=128, d_sae=512, k=8), model_name="gpt2", hook_name="blocks.1.hook_resid_pre",
        dataset_path="synthetic:uniform:500:32", context_size=16, training_tokens=256 * 10,
        train_batch_size_tokens=256, store_batch_size_prompts=8, n_batches_in_buffer=2,
        output_path=os.path.join(tmp, "out"), logger=LoggingConfig(log_to_wandb=False), device="cuda",
        save_mse_every_n_steps=1, n_checkpoints=0, verbose=False, streaming_mode=True,
        streaming_chunk_size_tokens=512, streaming_num_chunks=3, streaming_prefetch_chunks=1)
    runner = LanguageModelSAETrainingRunner(cfg, override_model=lm, vllm_dp_size=1)
    out = runner.run()
    info = {"role": runner.role, "transport": runner.streaming_transport}
    if runner.role == "consumer":
        info["steps"] = runner.trainer.n_training_steps
        info["engine"] = type(runner.trainer.engine).__name__
        info["d_sae"] = int(out.W_dec.shape[0])
    with open(os.path.join(tmp, f"r{rank}.json"), "w") as f:
        json.dump(info, f)
    dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_streaming_device_ring_runner(tmp_path):
    import torch.multiprocessing as mp

    mp.spawn(_worker, args=(2, _port(), str(tmp_path)), nprocs=2, join=True)
    p = json.loads((tmp_path / "r0.json").read_text())
    c = json.loads((tmp_path / "r1.json").read_text())
    assert p["role"] == "producer" and c["role"] == "consumer" and c["transport"] == "device"
    assert c["engine"] == "FusedTopKEngine" and c["steps"] == 10 and c["d_sae"] == 512
    out = tmp_path / "out"
    assert (out / "sae_weights.safetensors").exists()
    rows = [json.loads(x) for x in (out / "mse_history.jsonl").read_text().splitlines()]
    assert len(rows) == 10 and all(r["mse_loss"] == r["mse_loss"] for r in rows)
