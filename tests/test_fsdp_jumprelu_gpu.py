"""Sharded data-parallel native JumpReLU step (2 ranks: parameter all-gather fused into the encoder
GEMM with the JumpReLU epilogue, the weight-gradient reduce-scatter fused into the gradient GEMMs'
epilogues, sharded Adam including log_threshold) against the single-GPU dense JumpReLU step on the
concatenated batch, at the dense init of the reference's JumpReLU configs (threshold 0.001)."""

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


def _build(device):
    from saelens_b200.models.jumprelu import JumpReLUTrainingSAE, JumpReLUTrainingSAEConfig

    torch.manual_seed(7)
    sae = JumpReLUTrainingSAE(JumpReLUTrainingSAEConfig(d_in=256, d_sae=2048, jumprelu_init_threshold=0.001,
                                                        jumprelu_bandwidth=0.001, l0_coefficient=1.0,
                                                        device=device))
    with torch.no_grad():
        sae.b_enc.normal_(0, 0.01)
        sae.b_dec.normal_(0, 0.05)
    return sae


def _worker(rank, world, port, B, out_dir):
    import torch.distributed as dist
    from datetime import timedelta

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    from saelens_b200.parallel.fsdp_jumprelu_engine import FSDPJumpReLUEngine

    eng = FSDPJumpReLUEngine(_build(f"cuda:{rank}"), lr=1e-3, group=dist.group.WORLD)
    g = torch.Generator(device="cpu").manual_seed(11)
    x = torch.randn(B, 256, generator=g).to(torch.bfloat16)
    rows = x[rank * (B // world) : (rank + 1) * (B // world)].cuda()
    act = torch.zeros(2048, device=f"cuda:{rank}")
    eng.step(rows, update=False)
    torch.cuda.synchronize()
    g_dec, g_enc = eng.g_dec.float().cpu(), eng.g_enc.float().cpu()
    losses = [float(eng.step(rows, act_freq=act).loss) for _ in range(4)]
    torch.cuda.synchronize()
    eng.status.check()
    full = eng.full_weights()
    torch.save({"g_dec": g_dec, "g_enc": g_enc, "losses": losses, "act": act.cpu(),
                **{k: v.cpu() for k, v in full.items()}}, os.path.join(out_dir, f"rank{rank}.pt"))
    eng.close()
    dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_fsdp2_jumprelu_matches_single_gpu(tmp_path):
    import torch.multiprocessing as mp

    from saelens_b200.training.jumprelu_engine import JumpReLUEngine

    B = 512
    mp.spawn(_worker, args=(2, _free_port(), B, str(tmp_path)), nprocs=2, join=True)
    eng = JumpReLUEngine(_build("cuda:0"), lr=1e-3, mode="dense")
    g = torch.Generator(device="cpu").manual_seed(11)
    x = torch.randn(B, 256, generator=g).to(torch.bfloat16).cuda()
    act = torch.zeros(2048, device="cuda:0")
    eng.step(x, update=False)
    torch.cuda.synchronize()
    ref_g = {"g_dec": eng.g_dec.float().cpu(), "g_enc": eng.g_enc.float().cpu()}
    ref = [float(eng.step(x, act_freq=act).loss) for _ in range(4)]
    r = [torch.load(tmp_path / f"rank{i}.pt") for i in range(2)]
    for name in ("g_dec", "g_enc"):
        got = torch.cat([r[0][name], r[1][name]])
        rel = ((got - ref_g[name]).norm() / ref_g[name].norm()).item()
        assert rel < 1e-2, (name, rel)
    for a, b in zip(r[0]["losses"], ref):
        assert abs(a - b) <= 5e-3 * abs(b), (r[0]["losses"], ref)
    assert r[0]["losses"] == r[1]["losses"]
    assert torch.equal(r[0]["act"], r[1]["act"])
    assert (r[0]["act"] - act.cpu()).abs().sum() <= 1e-2 * act.sum().item()
    for i in range(2):
        for name, want in (("W_dec", eng.p_dec), ("W_enc", eng.p_enc.T), ("b_enc", eng.p_benc),
                           ("b_dec", eng.p_bdec), ("log_threshold", eng.p_lthr)):
            d = (r[i][name] - want.cpu()).abs()
            frac = (d > (2e-5 + 1e-3 * want.cpu().abs())).float().mean().item()
            assert d.max().item() <= 2 * 4 * 1e-3 and frac < 5e-2, (name, d.max().item(), frac)
