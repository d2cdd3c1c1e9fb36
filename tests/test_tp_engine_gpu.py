"""Tensor-parallel native step (2 ranks; fused NVLink kernels or NCCL exchanges) against the
single-GPU native step, with and without the dead-latent aux loss, for TopK and BatchTopK (the
batch-wide threshold is taken over the shards)."""

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


def _build(d_in, d_sae, k, device, kind="topk"):
    from saelens_b200.models.batchtopk import BatchTopKTrainingSAE, BatchTopKTrainingSAEConfig
    from saelens_b200.models.topk import TopKTrainingSAE, TopKTrainingSAEConfig

    torch.manual_seed(7)
    if kind == "batchtopk":
        sae = BatchTopKTrainingSAE(BatchTopKTrainingSAEConfig(d_in=d_in, d_sae=d_sae, k=k, device=device))
    else:
        sae = TopKTrainingSAE(TopKTrainingSAEConfig(d_in=d_in, d_sae=d_sae, k=k, device=device))
    with torch.no_grad():
        sae.b_enc.normal_(0, 0.01)
        sae.b_dec.normal_(0, 0.05)
    return sae


def _dead_mask(d_sae, device):
    return (torch.arange(d_sae, device=device) % 3) == 0


def _worker(rank, world, port, d_in, d_sae, k, B, out_dir, exchange, kind):
    import torch.distributed as dist
    from datetime import timedelta

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    from saelens_b200.parallel.tp_engine import TPTopKEngine

    sae = _build(d_in, d_sae, k, f"cuda:{rank}", kind)
    sae.shard_weights(dist.group.WORLD)
    eng = TPTopKEngine(sae, lr=1e-3, group=dist.group.WORLD, fused=exchange == "p2p")
    g = torch.Generator(device="cpu").manual_seed(11)
    x = torch.randn(B, d_in, generator=g).to(torch.bfloat16)
    rows = x[rank * (B // world) : (rank + 1) * (B // world)].cuda()
    n = d_sae // world
    dead = _dead_mask(d_sae, f"cuda:{rank}")[rank * n : (rank + 1) * n]
    losses = []
    for i in range(5):
        res = eng.step(rows, dead_mask=dead, run_aux=(i == 2))
        losses.append(float(res.loss))
    torch.cuda.synchronize()
    eng.status.check()
    eng.close()
    out = {"losses": losses, "p_dec": eng.p_dec.cpu(), "p_enc": eng.p_enc.cpu(), "p_bdec": eng.p_bdec.cpu()}
    if kind == "batchtopk":
        out["thr"] = float(sae.topk_threshold)
        out["truncated"] = int(eng.batch_truncated.item())
    torch.save(out, os.path.join(out_dir, f"rank{rank}.pt"))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("exchange,kind", [("p2p", "topk"), ("nccl", "topk"), ("p2p", "batchtopk"),
                                           ("nccl", "batchtopk")])
def test_tp2_matches_single_gpu(tmp_path, exchange, kind):
    import torch.multiprocessing as mp

    from saelens_b200.training.engine import FusedTopKEngine

    d_in, d_sae, k, B = 256, 2048, 32, 512
    mp.spawn(_worker, args=(2, _free_port(), d_in, d_sae, k, B, str(tmp_path), exchange, kind), nprocs=2,
             join=True)
    sae = _build(d_in, d_sae, k, "cuda:0", kind)
    eng = FusedTopKEngine(sae, lr=1e-3)
    g = torch.Generator(device="cpu").manual_seed(11)
    x = torch.randn(B, d_in, generator=g).to(torch.bfloat16).cuda()
    dead = _dead_mask(d_sae, "cuda:0")
    ref_losses = [float(eng.step(x, dead_mask=dead, run_aux=(i == 2)).loss) for i in range(5)]
    r = [torch.load(tmp_path / f"rank{i}.pt") for i in range(2)]
    for a, b in zip(r[0]["losses"], ref_losses):
        assert abs(a - b) <= 1e-3 * abs(b), (r[0]["losses"], ref_losses)
    assert r[0]["losses"] == r[1]["losses"]
    if kind == "batchtopk":
        # no row hit a candidate cap, so both runs select the same k*B entries
        assert int(eng.batch_truncated.item()) == 0 and r[0]["truncated"] == r[1]["truncated"] == 0
        want = float(sae.topk_threshold)
        assert want > 0 and r[0]["thr"] == r[1]["thr"]
        # the EMA of the smallest kept value; later steps' weights differ in their last bits
        assert abs(r[0]["thr"] - want) <= 1e-2 * want, (r[0]["thr"], want)
    n = d_sae // 2

    def close(got, want, name):
        # Adam normalises every coordinate, so a gradient that differs in its last bits (the TP
        # step sums partial reconstructions and gradient pairs in another order) can move a
        # near-zero coordinate by up to lr per step; everything else must agree tightly.
        d = (got - want).abs()
        bad = d > (2e-5 + 1e-3 * want.abs())
        frac = bad.float().mean().item()
        assert d.max().item() <= 5 * 1e-3 and frac < 2e-3, (name, d.max().item(), frac)

    for i in range(2):
        close(r[i]["p_dec"], eng.p_dec[i * n : (i + 1) * n].cpu(), f"p_dec{i}")
        close(r[i]["p_enc"], eng.p_enc[i * n : (i + 1) * n].cpu(), f"p_enc{i}")
        close(r[i]["p_bdec"], eng.p_bdec.cpu(), f"p_bdec{i}")
