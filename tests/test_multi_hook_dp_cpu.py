"""Multi-hook training with matched data parallelism on CPU (gloo, 2 ranks): each rank runs its
own LM on its dataset shard and trains one DDP-wrapped SAE per hook; replicas stay identical."""

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


def _worker(rank, world, port, tmp):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    import torch.distributed as dist

    dist.init_process_group("gloo", rank=rank, world_size=world)
    from saelens_b200.config import LanguageModelSAERunnerConfig, LoggingConfig
    from saelens_b200.models.lm import HookedLM, preset_config
    from saelens_b200.models.standard import StandardTrainingSAEConfig
    from saelens_b200.runners.llm_sae_training_runner import LanguageModelSAETrainingRunner

    torch.manual_seed(0)
    lm = HookedLM(preset_config("gpt2", n_layers=2, d_model=64, n_heads=4, d_mlp=128, d_vocab=500, n_ctx=64,
                                dtype="float32"))
    hooks = ["blocks.0.hook_resid_pre", "blocks.1.hook_resid_pre"]
    cfg = LanguageModelSAERunnerConfig(
        sae=StandardTrainingSAEConfig(d_in=64, d_sae=128, l1_coefficient=1e-3), model_name="gpt2",
        hook_names=hooks, dataset_path="synthetic:uniform:500:32", context_size=16, training_tokens=64 * 6,
        train_batch_size_tokens=64, store_batch_size_prompts=4, n_batches_in_buffer=2,
        output_path=os.path.join(tmp, "out"), logger=LoggingConfig(log_to_wandb=False), device="cpu",
        n_checkpoints=0, verbose=False, sae_dp_mode="ddp")
    runner = LanguageModelSAETrainingRunner(cfg, override_model=lm, vllm_dp_size=2, sae_dp_size=2)
    out = runner.run()
    with open(os.path.join(tmp, f"r{rank}.json"), "w") as f:
        json.dump({h: float(out[h].W_dec.detach().sum()) for h in hooks} | {"steps": runner.trainer.n_training_steps},
                  f)
    dist.destroy_process_group()


def test_multi_hook_matched_dp(tmp_path):
    mp.spawn(_worker, args=(2, _port(), str(tmp_path)), nprocs=2, join=True)
    r = [json.loads((tmp_path / f"r{i}.json").read_text()) for i in range(2)]
    assert r[0] == r[1] and r[0]["steps"] == 6
    assert (tmp_path / "out" / "multi_sae_manifest.json").exists() or any((tmp_path / "out").iterdir())
