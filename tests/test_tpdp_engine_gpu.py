"""Tensor x data parallel native step (TP=2 x DP=2 on 4 GPUs, fused P2P exchanges and P2P gradient
averaging) against the single-GPU native step on the whole batch."""

import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _build(d_in, d_sae, k, device):
    from saelens_b200.models.topk import TopKTrainingSAE, TopKTrainingSAEConfig

    torch.manual_seed(7)
    sae = TopKTrainingSAE(TopKTrainingSAEConfig(d_in=d_in, d_sae=d_sae, k=k, device=device))
    with torch.no_grad():
        sae.b_enc.normal_(0, 0.01)
        sae.b_dec.normal_(0, 0.05)
    return sae


def _worker(rank, world, port, d_in, d_sae, k, B, out_dir, tp_size):
    import torch.distributed as dist
    from datetime import timedelta

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    dp_size = world // tp_size
    tp_groups = [dist.new_group(list(range(d * tp_size, (d + 1) * tp_size))) for d in range(dp_size)]
    dp_groups = [dist.new_group(list(range(t, world, tp_size))) for t in range(tp_size)]
    tp_rank, dp_rank = rank % tp_size, rank // tp_size
    tp, dp = tp_groups[dp_rank], dp_groups[tp_rank]
    from saelens_b200.parallel.tp_engine import TPTopKEngine

    sae = _build(d_in, d_sae, k, f"cuda:{rank}")
    sae.shard_weights(tp)
    eng = TPTopKEngine(sae, lr=1e-3, group=tp, fused=True, dp_group=dp)
    g = torch.Generator(device="cpu").manual_seed(11)
    x = torch.randn(B, d_in, generator=g).to(torch.bfloat16)
    per_rep = B // dp_size
    rep = x[dp_rank * per_rep : (dp_rank + 1) * per_rep]
    rows = rep[tp_rank * (per_rep // tp_size) : (tp_rank + 1) * (per_rep // tp_size)].cuda()
    losses = [float(eng.step(rows).loss) for _ in range(3)]
    torch.cuda.synchronize()
    eng.status.check()
    torch.save({"losses": losses, "p_dec": eng.p_dec.cpu(), "p_bdec": eng.p_bdec.cpu()},
               os.path.join(out_dir, f"rank{rank}.pt"))
    eng.close()
    dist.destroy_process_group()


@pytest.mark.parametrize("tp_size,world", [(1, 2), (2, 4)])
def test_tp_dp_matches_single_gpu(tmp_path, tp_size, world):
    import torch.multiprocessing as mp

    from saelens_b200.training.engine import FusedTopKEngine

    if not torch.cuda.is_available() or torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    d_in, d_sae, k, B = 256, 2048, 32, 1024
    mp.spawn(_worker, args=(world, _free_port(), d_in, d_sae, k, B, str(tmp_path), tp_size), nprocs=world, join=True)
    sae = _build(d_in, d_sae, k, "cuda:0")
    eng = FusedTopKEngine(sae, lr=1e-3)
    g = torch.Generator(device="cpu").manual_seed(11)
    x = torch.randn(B, d_in, generator=g).to(torch.bfloat16).cuda()
    ref = [float(eng.step(x).loss) for _ in range(3)]
    r = [torch.load(tmp_path / f"rank{i}.pt") for i in range(world)]
    for a, b in zip(r[0]["losses"], ref):
        assert abs(a - b) <= 3e-3 * abs(b), (r[0]["losses"], ref)
    assert all(ri["losses"] == r[0]["losses"] for ri in r)
    for i in range(world):  # replicas of a shard stay identical
        assert torch.equal(r[i]["p_dec"], r[i % tp_size]["p_dec"])
    n = d_sae // tp_size
    for tp_rank in range(tp_size):
        got, want = r[tp_rank]["p_dec"], eng.p_dec[tp_rank * n : (tp_rank + 1) * n].cpu()
        d = (got - want).abs()
        frac = (d > (2e-5 + 1e-3 * want.abs())).float().mean().item()
        assert d.max().item() <= 2 * 3 * 1e-3 and frac < 5e-2, (tp_rank, d.max().item(), frac)
