"""Data-parallel native step (2 ranks, P2P gradient all-reduce) against the single-GPU native step
on the concatenated batch: averaging per-rank mean gradients equals the full-batch gradient."""

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


def _worker(rank, world, port, d_in, d_sae, k, B, out_dir, segments):
    import torch.distributed as dist
    from datetime import timedelta

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    from saelens_b200.parallel.ddp_engine import DDPTopKEngine

    sae = _build(d_in, d_sae, k, f"cuda:{rank}")
    eng = DDPTopKEngine(sae, lr=1e-3, group=dist.group.WORLD, segments=segments)
    g = torch.Generator(device="cpu").manual_seed(11)
    x = torch.randn(B, d_in, generator=g).to(torch.bfloat16)
    rows = x[rank * (B // world) : (rank + 1) * (B // world)].cuda()
    act = torch.zeros(d_sae, device=f"cuda:{rank}")
    since = torch.zeros(d_sae, device=f"cuda:{rank}")
    eng.step(rows, update=False)  # gradient only: the averaged gradient is compared directly
    torch.cuda.synchronize()
    g0 = {"g_dec": eng.g_avg[0].float().cpu(), "g_enc": eng.g_avg[1].float().cpu()}
    losses = []
    for _ in range(4):
        losses.append(float(eng.step(rows, act_freq=act, since_fired=since).loss))
    torch.cuda.synchronize()
    eng.status.check()
    torch.save({"losses": losses, "p_dec": eng.p_dec.cpu(), "p_enc": eng.p_enc.cpu(), "p_bdec": eng.p_bdec.cpu(),
                "act": act.cpu(), "since": since.cpu(), **g0}, os.path.join(out_dir, f"rank{rank}.pt"))
    eng.close()
    dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("segments", [1, 3])
def test_ddp2_matches_single_gpu_full_batch(tmp_path, segments):
    import torch.multiprocessing as mp

    from saelens_b200.training.engine import FusedTopKEngine

    d_in, d_sae, k, B = 256, 2048, 32, 512
    mp.spawn(_worker, args=(2, _free_port(), d_in, d_sae, k, B, str(tmp_path), segments), nprocs=2, join=True)
    sae = _build(d_in, d_sae, k, "cuda:0")
    eng = FusedTopKEngine(sae, lr=1e-3)
    g = torch.Generator(device="cpu").manual_seed(11)
    x = torch.randn(B, d_in, generator=g).to(torch.bfloat16).cuda()
    act = torch.zeros(d_sae, device="cuda:0")
    since = torch.zeros(d_sae, device="cuda:0")
    eng.step(x, update=False)
    torch.cuda.synchronize()
    live = (eng.colptr[1:] > eng.colptr[:-1]).cpu()
    ref_g = {"g_dec": eng.g_dec.float().cpu(), "g_enc": eng.g_enc.float().cpu()}
    ref = [float(eng.step(x, act_freq=act, since_fired=since).loss) for _ in range(4)]
    r = [torch.load(tmp_path / f"rank{i}.pt") for i in range(2)]
    # the averaged gradient equals the full-batch gradient up to bf16 rounding of the per-rank parts
    for name in ("g_dec", "g_enc"):
        got, want = r[0][name], ref_g[name]
        assert torch.equal(r[0][name], r[1][name])
        assert got[~live].abs().max().item() == 0.0 if (~live).any() else True
        rel = ((got[live] - want[live]).norm() / want[live].norm()).item()
        assert rel < 1e-2, (name, rel)
    for a, b in zip(r[0]["losses"], ref):
        assert abs(a - b) <= 2e-3 * abs(b), (r[0]["losses"], ref)
    assert r[0]["losses"] == r[1]["losses"]
    # replicas stay identical without any parameter broadcast
    for name in ("p_dec", "p_enc", "p_bdec"):
        assert torch.equal(r[0][name], r[1][name]), name
    # firing statistics cover the global batch (equal up to selections that flip on near-ties once
    # the two runs' parameters differ in their last bits)
    assert torch.equal(r[0]["act"], r[1]["act"])
    assert (r[0]["act"] - act.cpu()).abs().sum().item() <= 1e-3 * act.sum().item()
    assert (r[0]["since"] != since.cpu()).float().mean().item() < 1e-2

    def close(got, want, name):
        # Adam normalises each coordinate, so coordinates whose gradient is near zero can move in
        # opposite directions by up to lr per step between the two runs; the bulk must agree
        d = (got - want).abs()
        frac = (d > (2e-5 + 1e-3 * want.abs())).float().mean().item()
        assert d.max().item() <= 2 * 4 * 1e-3 and frac < 5e-2, (name, d.max().item(), frac)

    close(r[0]["p_dec"], eng.p_dec.cpu(), "p_dec")
    close(r[0]["p_enc"], eng.p_enc.cpu(), "p_enc")
    close(r[0]["p_bdec"], eng.p_bdec.cpu(), "p_bdec")
