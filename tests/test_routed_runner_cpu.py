"""Shard-routing mode of the LM training runner on CPU (gloo, collective transport): a disjoint
producer -> consumer pair, and two co-located producer+consumer ranks training one SAE with
data parallelism."""

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


def _worker(rank, world, port, tmp, P, Q, tp=1, vtp=1, hooks=None):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    import torch.distributed as dist

    dist.init_process_group("gloo", rank=rank, world_size=world)
    from saelens_b200.config import LanguageModelSAERunnerConfig, LoggingConfig
    from saelens_b200.models.lm import HookedLM, preset_config
    from saelens_b200.models.standard import StandardTrainingSAEConfig
    from saelens_b200.models.topk import TopKTrainingSAEConfig
    from saelens_b200.runners.llm_sae_training_runner import LanguageModelSAETrainingRunner

    torch.manual_seed(0)
    lm = HookedLM(preset_config("gpt2", n_layers=2, d_model=64, n_heads=4, d_mlp=128, d_vocab=500, n_ctx=64,
                                dtype="float32"))
    torch.manual_seed(1)
    cfg = LanguageModelSAERunnerConfig(
        sae=(StandardTrainingSAEConfig(d_in=64, d_sae=128, l1_coefficient=1e-3) if tp == 1
             else TopKTrainingSAEConfig(d_in=64, d_sae=128, k=8)), model_name="gpt2",
        hook_name="blocks.1.hook_resid_pre", dataset_path="synthetic:uniform:500:32", context_size=16,
        training_tokens=64 * 8, train_batch_size_tokens=64, store_batch_size_prompts=4, n_batches_in_buffer=2,
        output_path=os.path.join(tmp, "out"), logger=LoggingConfig(log_to_wandb=False), device="cpu",
        save_mse_every_n_steps=1, n_checkpoints=0, verbose=False, routing_transport="collective",
        **({"hook_names": list(hooks)} if hooks else {}))
    if rank == 1:  # a rank with other paths (e.g. another timestamp) follows rank 0
        cfg.checkpoint_path = os.path.join(tmp, "elsewhere")
    runner = LanguageModelSAETrainingRunner(cfg, override_model=lm, vllm_dp_size=P, sae_dp_size=Q,
                                            sae_tp_size=tp, vllm_tp_size=vtp, use_shard_routing=True)
    assert cfg.checkpoint_path != os.path.join(tmp, "elsewhere")
    out = runner.run()
    info = {"role": runner.role, "transport": runner.routing_transport,
            "lm_sharded": getattr(runner.model, "tp", None) is not None}
    if isinstance(out, dict):
        info["steps"] = runner.trainer.n_training_steps
        info["W_dec_sum"] = {h: float(s.W_dec.detach().sum()) for h, s in out.items()}
    elif out is not None:
        info["steps"] = runner.trainer.n_training_steps
        info["W_dec_sum"] = float(out.W_dec.detach().sum())
    with open(os.path.join(tmp, f"r{rank}.json"), "w") as f:
        json.dump(info, f)
    dist.destroy_process_group()


@pytest.mark.parametrize("P,Q", [(1, 1), (2, 2)])
def test_routed_runner(tmp_path, P, Q):
    mp.spawn(_worker, args=(2, _port(), str(tmp_path), P, Q), nprocs=2, join=True)
    r = [json.loads((tmp_path / f"r{i}.json").read_text()) for i in range(2)]
    if (P, Q) == (1, 1):
        assert r[0]["role"] == "producer" and r[1]["role"] == "consumer"
        assert r[1]["steps"] == 8 and r[1]["transport"] == "collective"
    else:
        assert r[0]["role"] == r[1]["role"] == "producer+consumer"
        assert r[0]["steps"] == r[1]["steps"] == 8
        assert r[0]["W_dec_sum"] == pytest.approx(r[1]["W_dec_sum"], rel=1e-6)  # DP replicas agree
    assert (tmp_path / "out" / "sae_weights.safetensors").exists()


def test_routed_runner_to_tensor_parallel_consumer(tmp_path):
    """One producer feeds an SAE whose latents are sharded over two consumer ranks: the consumer
    root receives the rows and broadcasts them to its TP member."""
    mp.spawn(_worker, args=(3, _port(), str(tmp_path), 1, 1, 2), nprocs=3, join=True)
    r = [json.loads((tmp_path / f"r{i}.json").read_text()) for i in range(3)]
    assert r[0]["role"] == "producer" and r[1]["role"] == r[2]["role"] == "consumer"
    assert r[1]["steps"] == r[2]["steps"] == 8


def test_routed_runner_with_tensor_parallel_producer(tmp_path):
    """A producer whose LM is split over two ranks (Megatron TP, every member runs its shard, the
    first rank sends) trains the consumer's SAE exactly as a one-rank producer does."""
    mp.spawn(_worker, args=(3, _port(), str(tmp_path / "tp"), 1, 1, 1, 2), nprocs=3, join=True)
    r = [json.loads((tmp_path / "tp" / f"r{i}.json").read_text()) for i in range(3)]
    assert r[0]["role"] == r[1]["role"] == "producer" and r[2]["role"] == "consumer"
    assert r[0]["lm_sharded"] and r[1]["lm_sharded"] and r[2]["steps"] == 8
    mp.spawn(_worker, args=(2, _port(), str(tmp_path / "one"), 1, 1), nprocs=2, join=True)
    one = json.loads((tmp_path / "one" / "r1.json").read_text())
    assert r[2]["W_dec_sum"] == pytest.approx(one["W_dec_sum"], rel=1e-4, abs=1e-4)


def _resume_worker(rank, world, port, tmp, phase):
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
    cfg = LanguageModelSAERunnerConfig(
        sae=StandardTrainingSAEConfig(d_in=64, d_sae=128, l1_coefficient=1e-3), model_name="gpt2",
        hook_name="blocks.1.hook_resid_pre", dataset_path="synthetic:uniform:500:32", context_size=16,
        training_tokens=64 * 8, train_batch_size_tokens=64, store_batch_size_prompts=4, n_batches_in_buffer=2,
        output_path=os.path.join(tmp, f"out{phase}"), checkpoint_path=os.path.join(tmp, "ckpt"),
        logger=LoggingConfig(log_to_wandb=False), device="cpu", n_checkpoints=1, save_final_checkpoint=False,
        verbose=False, routing_transport="collective")
    resume = None
    if phase == 2:  # the config adds a run id under checkpoint_path
        from pathlib import Path

        resume = str(next(Path(tmp, "ckpt").glob("*/320")))
    runner = LanguageModelSAETrainingRunner(cfg, override_model=lm, vllm_dp_size=1, sae_dp_size=1,
                                            use_shard_routing=True, resume_from_checkpoint=resume)
    runner.run()
    if runner.role == "consumer":
        with open(os.path.join(tmp, f"steps{phase}.json"), "w") as f:
            json.dump({"samples": runner.trainer.n_training_samples,
                       "mse_rows": len(runner.trainer.mse_history_path.read_text().splitlines())
                       if runner.trainer.mse_history_path else None}, f)
    dist.destroy_process_group()


def test_routed_runner_checkpoint_and_resume(tmp_path):
    mp.spawn(_resume_worker, args=(2, _port(), str(tmp_path), 1), nprocs=2, join=True)
    ck = next((tmp_path / "ckpt").glob("*/320"))
    assert (ck / "trainer_state.pt").exists() and (ck / "producer_dataset_state_0").exists()
    mp.spawn(_resume_worker, args=(2, _port(), str(tmp_path), 2), nprocs=2, join=True)
    # the resumed run trains the 3 remaining steps (samples 320 -> 512); the producer sends exactly
    # those, so nothing waits on a send that is never received
    st = json.loads((tmp_path / "steps2.json").read_text())
    assert st["samples"] == 512
    assert (tmp_path / "out2" / "sae_weights.safetensors").exists()


def _colocated_tp_worker(rank, world, port, tmp):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    import torch.distributed as dist

    dist.init_process_group("gloo", rank=rank, world_size=world)
    from saelens_b200.config import LanguageModelSAERunnerConfig, LoggingConfig
    from saelens_b200.models.batchtopk import BatchTopKTrainingSAEConfig
    from saelens_b200.models.lm import HookedLM, preset_config
    from saelens_b200.runners.llm_sae_training_runner import LanguageModelSAETrainingRunner

    torch.manual_seed(0)
    lm = HookedLM(preset_config("gpt2", n_layers=2, d_model=64, n_heads=4, d_mlp=128, d_vocab=500, n_ctx=64,
                                dtype="float32"))
    cfg = LanguageModelSAERunnerConfig(
        sae=BatchTopKTrainingSAEConfig(d_in=64, d_sae=128, k=8), model_name="gpt2",
        hook_name="blocks.1.hook_resid_pre", dataset_path="synthetic:uniform:500:32", context_size=16,
        training_tokens=64 * 6, train_batch_size_tokens=64, store_batch_size_prompts=4, n_batches_in_buffer=2,
        output_path=os.path.join(tmp, "out"), logger=LoggingConfig(log_to_wandb=False), device="cpu",
        n_checkpoints=0, verbose=False, routing_transport="collective", sae_dp_mode="manual")
    runner = LanguageModelSAETrainingRunner(cfg, override_model=lm, vllm_dp_size=2, sae_dp_size=2, sae_tp_size=2,
                                            use_shard_routing=True)
    out = runner.run()
    info = {"role": runner.role}
    if out is not None:
        info["steps"] = runner.trainer.n_training_steps
        info["W_dec_shard_rows"] = int(out.W_dec.shape[0])
    with open(os.path.join(tmp, f"r{rank}.json"), "w") as f:
        json.dump(info, f)
    dist.destroy_process_group()


def test_routed_colocated_producers_with_tp_dp_consumers(tmp_path):
    """2 producers co-located with the first ranks of two data-parallel SAE replicas of TP 2."""
    mp.spawn(_colocated_tp_worker, args=(4, _port(), str(tmp_path)), nprocs=4, join=True)
    r = [json.loads((tmp_path / f"r{i}.json").read_text()) for i in range(4)]
    assert [x["role"] for x in r] == ["producer+consumer", "producer+consumer", "consumer", "consumer"]
    assert all(x["steps"] == 6 and x["W_dec_shard_rows"] == 64 for x in r)


@pytest.mark.parametrize("P,Q", [(1, 1), (2, 2)])
def test_routed_runner_multi_hook(tmp_path, P, Q):
    """Two hooks routed side by side in one row: every consumer trains one SAE per hook, data
    parallel replicas stay equal, and the final SAEs are written one directory per hook."""
    hooks = ["blocks.0.hook_resid_pre", "blocks.1.hook_resid_pre"]
    mp.spawn(_worker, args=(2, _port(), str(tmp_path), P, Q, 1, 1, hooks), nprocs=2, join=True)
    r = [json.loads((tmp_path / f"r{i}.json").read_text()) for i in range(2)]
    trained = [x for x in r if "steps" in x]
    assert trained and all(x["steps"] == 8 for x in trained)
    assert all(set(x["W_dec_sum"]) == set(hooks) for x in trained)
    if (P, Q) == (2, 2):
        for h in hooks:
            assert r[0]["W_dec_sum"][h] == pytest.approx(r[1]["W_dec_sum"][h], rel=1e-6)
    sums = trained[0]["W_dec_sum"]
    assert sums[hooks[0]] != sums[hooks[1]]  # each hook's SAE trained on its own activations
    subdirs = [p for p in (tmp_path / "out").iterdir() if p.is_dir()]
    assert len(subdirs) == 2 and all((d / "sae_weights.safetensors").exists() for d in subdirs)
