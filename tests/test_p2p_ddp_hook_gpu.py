"""DDP with the P2P all-reduce communication hook against DDP's own NCCL all-reduce (2 ranks):
gradients after each backward and parameters after Adam steps are identical (a sum of two fp32
values and the 1/2 scale are exact in any order)."""

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


def _worker(rank, world, port, out_dir, dtype_name):
    import torch.distributed as dist
    from datetime import timedelta

    from torch.nn.parallel import DistributedDataParallel as DDP

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    from saelens_b200.models.standard import StandardTrainingSAE, StandardTrainingSAEConfig
    from saelens_b200.parallel.p2p_ddp_hook import p2p_hook_supported, register_p2p_allreduce

    dtype = getattr(torch, dtype_name)

    def build():
        torch.manual_seed(5)
        return StandardTrainingSAE(StandardTrainingSAEConfig(d_in=256, d_sae=1024, device=f"cuda:{rank}",
                                                             dtype=dtype_name))

    sa, sb = build(), build()
    assert p2p_hook_supported(sa, dist.group.WORLD)
    da = DDP(sa, device_ids=[rank], bucket_cap_mb=0.25)  # several buckets
    db = DDP(sb, device_ids=[rank], bucket_cap_mb=0.25)
    state = register_p2p_allreduce(da, sa, dist.group.WORLD, 0.25)
    oa = torch.optim.Adam(sa.parameters(), lr=1e-3)
    ob = torch.optim.Adam(sb.parameters(), lr=1e-3)
    same_grads = []
    for step in range(4):
        g = torch.Generator(device="cpu").manual_seed(100 * step + rank)
        x = torch.randn(64, 256, generator=g).to(dtype).cuda()
        for d, o in ((da, oa), (db, ob)):
            o.zero_grad()
            y = d(x)
            ((y.float() - x.float()) ** 2).sum().backward()
        same_grads.append(all(torch.equal(pa.grad, pb.grad) for pa, pb in zip(sa.parameters(), sb.parameters())))
        oa.step()
        ob.step()
    torch.cuda.synchronize()
    state.check()
    same_params = all(torch.equal(pa, pb) for pa, pb in zip(sa.parameters(), sb.parameters()))
    torch.save({"grads": same_grads, "params": same_params, "calls": state.calls, "shapes": len(state.areas),
                "fallbacks": state.nccl_fallbacks},
               os.path.join(out_dir, f"r{rank}.pt"))
    state.close()
    dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("dtype_name", ["float32", "bfloat16"])
def test_p2p_ddp_hook_matches_nccl(tmp_path, dtype_name):
    import torch.multiprocessing as mp

    mp.spawn(_worker, args=(2, _free_port(), str(tmp_path), dtype_name), nprocs=2, join=True)
    for r in range(2):
        res = torch.load(tmp_path / f"r{r}.pt")
        assert all(res["grads"]) and res["params"], res
        assert res["calls"] >= 4 and res["shapes"] >= 1 and res["fallbacks"] == 0, res
