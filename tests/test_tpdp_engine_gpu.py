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


def _worker(rank, world, port, d_in, d_sae, k, B, out_dir):
    import torch.distributed as dist
    from datetime import timedelta

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    tp_groups = [dist.new_group([0, 1]), dist.new_group([2, 3])]
    dp_groups = [dist.new_group([0, 2]), dist.new_group([1, 3])]
    tp_rank, dp_rank = rank % 2, rank // 2
    tp, dp = tp_groups[dp_rank], dp_groups[tp_rank]
    from saelens_b200.parallel.tp_engine import TPTopKEngine

    sae = _build(d_in, d_sae, k, f"cuda:{rank}")
    sae.shard_weights(tp)
    eng = TPTopKEngine(sae, lr=1e-3, group=tp, fused=True, dp_group=dp)
    g = torch.Generator(device="cpu").manual_seed(11)
    x = torch.randn(B, d_in, generator=g).to(torch.bfloat16)
    rep = x[dp_rank * (B // 2) : (dp_rank + 1) * (B // 2)]
    rows = rep[tp_rank * (B // 4) : (tp_rank + 1) * (B // 4)].cuda()
    losses = [float(eng.step(rows).loss) for _ in range(3)]
    torch.cuda.synchronize()
    eng.status.check()
    torch.save({"losses": losses, "p_dec": eng.p_dec.cpu(), "p_bdec": eng.p_bdec.cpu()},
               os.path.join(out_dir, f"rank{rank}.pt"))
    eng.close()
    dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 4, reason="needs 4 GPUs")
def test_tp2_dp2_matches_single_gpu(tmp_path):
    import torch.multiprocessing as mp

    from saelens_b200.training.engine import FusedTopKEngine

    d_in, d_sae, k, B = 256, 2048, 32, 1024
    mp.spawn(_worker, args=(4, _free_port(), d_in, d_sae, k, B, str(tmp_path)), nprocs=4, join=True)
    sae = _build(d_in, d_sae, k, "cuda:0")
    eng = FusedTopKEngine(sae, lr=1e-3)
    g = torch.Generator(device="cpu").manual_seed(11)
    x = torch.randn(B, d_in, generator=g).to(torch.bfloat16).cuda()
    ref = [float(eng.step(x).loss) for _ in range(3)]
    r = [torch.load(tmp_path / f"rank{i}.pt") for i in range(4)]
    for a, b in zip(r[0]["losses"], ref):
        assert abs(a - b) <= 3e-3 * abs(b), (r[0]["losses"], ref)
    assert r[0]["losses"] == r[1]["losses"] == r[2]["losses"] == r[3]["losses"]
    assert torch.equal(r[0]["p_dec"], r[2]["p_dec"]) and torch.equal(r[1]["p_dec"], r[3]["p_dec"])
    n = d_sae // 2
    for tp_rank in range(2):
        got, want = r[tp_rank]["p_dec"], eng.p_dec[tp_rank * n : (tp_rank + 1) * n].cpu()
        d = (got - want).abs()
        frac = (d > (2e-5 + 1e-3 * want.abs())).float().mean().item()
        assert d.max().item() <= 2 * 3 * 1e-3 and frac < 5e-2, (tp_rank, d.max().item(), frac)
