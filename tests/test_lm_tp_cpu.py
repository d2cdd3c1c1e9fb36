"""Producer tensor parallelism on CPU (gloo, 2 ranks): the Megatron-split LM gives, for every
hook name (residual stream, attention q / k / v / z, rotated q / k, MLP pre / post), the same
capture as the unsplit model, on every rank."""

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


HOOKS = ["blocks.0.hook_resid_pre", "blocks.0.attn.hook_q", "blocks.0.attn.hook_k", "blocks.0.attn.hook_v",
         "blocks.0.attn.hook_rot_q", "blocks.1.attn.hook_z", "blocks.1.hook_attn_out", "blocks.1.hook_resid_mid",
         "blocks.1.mlp.hook_pre", "blocks.1.mlp.hook_post", "blocks.1.hook_mlp_out", "blocks.1.hook_resid_post"]


def _model(preset):
    from saelens_b200.models.lm.transformer import HookedLM, preset_config

    over = dict(n_layers=2, d_model=64, n_heads=4, d_mlp=128, d_vocab=300, n_ctx=32, dtype="float32")
    if preset != "gpt2":
        over["n_key_value_heads"] = 2
    torch.manual_seed(0)
    return HookedLM(preset_config(preset, **over))


def _worker(rank, world, port, preset, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import torch.distributed as dist

    dist.init_process_group("gloo", rank=rank, world_size=world)
    from saelens_b200.models.lm.tp import shard_lm_tensor_parallel

    toks = torch.randint(0, 300, (2, 12), generator=torch.Generator().manual_seed(1))
    hooks = [h for h in HOOKS if not (preset == "gpt2" and "rot_q" in h)]
    full = _model(preset)
    with torch.no_grad():
        ref_logits, ref = full.run_with_cache(toks, names_filter=hooks)
    tp = shard_lm_tensor_parallel(_model(preset), dist.group.WORLD)
    with torch.no_grad():
        logits, got = tp.run_with_cache(toks, names_filter=hooks)
    errs = {h: (got[h] - ref[h]).abs().max().item() for h in hooks}
    errs["logits"] = (logits - ref_logits).abs().max().item()
    shapes = {h: tuple(got[h].shape) == tuple(ref[h].shape) for h in hooks}
    torch.save({"errs": errs, "shapes": shapes, "gathers": tp.tp.gathers}, os.path.join(out, f"r{rank}.pt"))
    dist.destroy_process_group()


@pytest.mark.parametrize("preset", ["llama-3-8b", "gpt2"])
def test_tp2_capture_equals_tp1_for_every_hook(tmp_path, preset):
    mp.spawn(_worker, args=(2, _port(), preset, str(tmp_path)), nprocs=2, join=True)
    for rank in range(2):
        r = torch.load(tmp_path / f"r{rank}.pt")
        assert all(r["shapes"].values()), r["shapes"]
        assert max(r["errs"].values()) < 1e-4, r["errs"]
        assert r["gathers"] > 0
