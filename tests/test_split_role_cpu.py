"""Split-role data path (local overlap with SAE tensor parallelism, gloo, 2 ranks): only the
replica's LM root runs the language model and broadcasts each batch to its SAE TP group; the TP
run matches a single-process run on the same tokens."""

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


def _cfg(tmp, name):
    from saelens_b200.config import LanguageModelSAERunnerConfig, LoggingConfig
    from saelens_b200.models.topk import TopKTrainingSAEConfig

    return LanguageModelSAERunnerConfig(
        sae=TopKTrainingSAEConfig(d_in=64, d_sae=256, k=8), model_name="gpt2",
        hook_name="blocks.1.hook_resid_pre", dataset_path="synthetic:uniform:500:16", context_size=16,
        training_tokens=64 * 5, train_batch_size_tokens=64, store_batch_size_prompts=4, n_batches_in_buffer=2,
        output_path=os.path.join(tmp, name), logger=LoggingConfig(log_to_wandb=False), device="cpu",
        n_checkpoints=0, verbose=False, lr=1e-3, seed=3)


def _lm():
    from saelens_b200.models.lm import HookedLM, preset_config

    torch.manual_seed(0)
    return HookedLM(preset_config("gpt2", n_layers=2, d_model=64, n_heads=4, d_mlp=128, d_vocab=500, n_ctx=64,
                                  dtype="float32"))


def _worker(rank, world, port, tmp):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    import torch.distributed as dist

    dist.init_process_group("gloo", rank=rank, world_size=world)
    from saelens_b200.runners.llm_sae_training_runner import LanguageModelSAETrainingRunner

    lm = _lm()
    runner = LanguageModelSAETrainingRunner(_cfg(tmp, "tp"), override_model=lm, sae_tp_size=2)
    info = {"role": runner.role, "has_model": runner.model is not None,
            "has_store": runner.activations_store is not None}
    runner.run()
    info["steps"] = runner.trainer.n_training_steps
    with open(os.path.join(tmp, f"r{rank}.json"), "w") as f:
        json.dump(info, f)
    dist.barrier()
    dist.destroy_process_group()


def test_split_role_tp2_matches_single_process(tmp_path):
    from safetensors.torch import load_file

    from saelens_b200.runners.llm_sae_training_runner import LanguageModelSAETrainingRunner

    mp.spawn(_worker, args=(2, _port(), str(tmp_path)), nprocs=2, join=True)
    r = [json.loads((tmp_path / f"r{i}.json").read_text()) for i in range(2)]
    assert r[0] == {"role": "producer+consumer", "has_model": True, "has_store": True, "steps": 5}
    assert r[1] == {"role": "consumer", "has_model": False, "has_store": False, "steps": 5}
    single = LanguageModelSAETrainingRunner(_cfg(str(tmp_path), "single"), override_model=_lm())
    single.run()
    a = load_file(str(tmp_path / "tp" / "sae_weights.safetensors"))
    b = load_file(str(tmp_path / "single" / "sae_weights.safetensors"))
    for key in ("W_enc", "W_dec", "b_enc", "b_dec"):
        torch.testing.assert_close(a[key], b[key], atol=1e-5, rtol=1e-4)
