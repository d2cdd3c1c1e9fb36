"""Streaming mode of the LM training runner on CPU (gloo, 2 ranks, host ring): rank 0 runs the LM
and writes activation chunks, rank 1 trains the SAE from the ring and saves it."""

import json
import os
import socket

import torch
import torch.multiprocessing as mp


def _port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, tmp, vtp=1, stp=1, hooks=None):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    import torch.distributed as dist

    dist.init_process_group("gloo", rank=rank, world_size=world)
    from saelens_b200.config import LanguageModelSAERunnerConfig, LoggingConfig
    from saelens_b200.models.lm import HookedLM, preset_config
    from saelens_b200.models.topk import TopKTrainingSAEConfig
    from saelens_b200.runners.llm_sae_training_runner import LanguageModelSAETrainingRunner

    torch.manual_seed(0)
    lm = HookedLM(preset_config("gpt2", n_layers=2, d_model=64, n_heads=4, d_mlp=128, d_vocab=500, n_ctx=64,
                                dtype="float32"))
    cfg = LanguageModelSAERunnerConfig(
        sae=TopKTrainingSAEConfig(d_in=64, d_sae=128, k=8), model_name="gpt2", hook_name="blocks.1.hook_resid_pre",
        hook_names=hooks,
        dataset_path="synthetic:uniform:500:32", context_size=16, training_tokens=64 * 12,
        train_batch_size_tokens=64, store_batch_size_prompts=4, n_batches_in_buffer=2,
        output_path=os.path.join(tmp, "out"), logger=LoggingConfig(log_to_wandb=False), device="cpu",
        save_mse_every_n_steps=1, n_checkpoints=0, verbose=False, streaming_mode=True,
        streaming_chunk_size_tokens=128, streaming_num_chunks=4, streaming_prefetch_chunks=1,
        streaming_buffer_name=f"ring_{port}", streaming_buffer_dir=tmp, streaming_transport="host")
    if rank == 0:  # the ring's files are created before the runners attach
        from saelens_b200.training.shared_activation_buffer import SharedActivationBuffer

        SharedActivationBuffer(f"ring_{port}", 4, 128 * (len(hooks) if hooks else 1), 64, num_producers=1,
                               target_chunks=6, create=True, base_dir=tmp, dtype=torch.float32).close()
    dist.barrier()
    runner = LanguageModelSAETrainingRunner(cfg, override_model=lm, vllm_dp_size=1, vllm_tp_size=vtp, sae_tp_size=stp)
    out = runner.run()
    info = {"role": runner.role, "transport": runner.streaming_transport,
            "lm_sharded": getattr(runner.model, "tp", None) is not None}
    if runner.role == "consumer" and hooks:
        info["steps"] = runner.trainer.n_training_steps
        info["hooks"] = sorted(out.keys())
    elif runner.role == "consumer":
        info["steps"] = runner.trainer.n_training_steps
        info["d_sae"] = int(out.W_dec.shape[0])
        info["d_sae_local"] = int(runner.sae.W_dec.shape[0])
    with open(os.path.join(tmp, f"r{rank}.json"), "w") as f:
        json.dump(info, f)
    dist.destroy_process_group()


def test_streaming_host_ring_producer_to_consumer(tmp_path):
    mp.spawn(_worker, args=(2, _port(), str(tmp_path)), nprocs=2, join=True)
    p = json.loads((tmp_path / "r0.json").read_text())
    c = json.loads((tmp_path / "r1.json").read_text())
    assert p["role"] == "producer" and c["role"] == "consumer" and c["transport"] == "host"
    assert c["steps"] == 12 and c["d_sae"] == 128  # 6 chunks x 128 rows / 64 rows per step
    out = tmp_path / "out"
    assert (out / "cfg.json").exists() and (out / "sae_weights.safetensors").exists()
    rows = [json.loads(x) for x in (out / "mse_history.jsonl").read_text().splitlines()]
    assert len(rows) == 12


def test_streaming_with_tensor_parallel_producer(tmp_path):
    """The producer's LM split over two ranks (Megatron TP): both run every forward, the first rank
    writes the chunks; the consumer trains the same number of steps."""
    mp.spawn(_worker, args=(3, _port(), str(tmp_path), 2), nprocs=3, join=True)
    r = [json.loads((tmp_path / f"r{i}.json").read_text()) for i in range(3)]
    assert r[0]["role"] == r[1]["role"] == "producer" and r[0]["lm_sharded"] and r[1]["lm_sharded"]
    assert r[2]["role"] == "consumer" and r[2]["steps"] == 12


def test_streaming_consumer_is_sae_tensor_parallel(tmp_path):
    """Two consumer ranks form the SAE TP group: each trains its latent shard of the SAE, both train
    every step, and the saved SAE is the gathered full dictionary (one timing / MSE writer)."""
    mp.spawn(_worker, args=(3, _port(), str(tmp_path), 1, 2), nprocs=3, join=True)
    r = [json.loads((tmp_path / f"r{i}.json").read_text()) for i in range(3)]
    assert r[0]["role"] == "producer" and r[1]["role"] == r[2]["role"] == "consumer"
    assert r[1]["d_sae_local"] == r[2]["d_sae_local"] == 64 and r[1]["steps"] == r[2]["steps"] == 12
    out = tmp_path / "out"
    rows = [json.loads(x) for x in (out / "mse_history.jsonl").read_text().splitlines()]
    assert len(rows) == 12


def test_streaming_multi_hook_trains_one_sae_per_hook(tmp_path):
    """Two hooks through the ring (per training step one block of rows per hook): the consumer
    trains one SAE per hook for every step and writes both SAEs and the manifest."""
    hooks = ["blocks.0.hook_resid_post", "blocks.1.hook_resid_pre"]
    mp.spawn(_worker, args=(2, _port(), str(tmp_path), 1, 1, hooks), nprocs=2, join=True)
    c = json.loads((tmp_path / "r1.json").read_text())
    assert c["role"] == "consumer" and c["steps"] == 12 and c["hooks"] == sorted(hooks)
    out = tmp_path / "out"
    assert (out / "multi_sae_manifest.json").exists()
    for h in hooks:
        assert (out / h / "sae_weights.safetensors").exists() and (out / h / "cfg.json").exists()
