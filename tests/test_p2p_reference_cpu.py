"""CPU tier for every peer-memory collective algorithm: the reference implementations on gloo
ranks (world sizes 2 and 3) against single-process formulas."""

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


def _worker(rank, world, port, out_dir):
    import torch.distributed as dist

    from saelens_b200.parallel import p2p_reference as R

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    res = {}
    g = torch.Generator().manual_seed(rank)
    # two-shot all-reduce with a ragged tail chunk, bf16 and fp32
    x = torch.randn(10_000, generator=g)
    res["ar_f32"], res["ar_f32_sq"] = R.two_shot_allreduce(x, chunk=2048, scale=0.5)
    res["ar_bf16"], _ = R.two_shot_allreduce(x.to(torch.bfloat16), chunk=4096)
    # decode reduce-scatter
    B, D = 6 * world, 8
    partial = torch.randn(B, D, generator=g)
    b_dec = torch.ones(D)
    tgt_all = torch.randn(B, D, generator=torch.Generator().manual_seed(99))
    Bo = B // world
    res["rs"] = R.decode_reduce_scatter(partial, b_dec, tgt_all[rank * Bo : (rank + 1) * Bo], 2.0 / B)
    res["partial"] = partial
    # candidate merge: k=3 candidates per row from each rank, shared ties
    vals = torch.tensor([[5.0, 3.0, 1.0], [2.0, 2.0, 0.5]])
    idx = torch.tensor([[0, 1, 2], [3, 4, -1]])
    res["keep"] = R.candidate_merge(vals, idx, n_local=10, k=3)
    # row routing: rank 0 produces, the others consume
    xr = torch.randn(12, 4, generator=torch.Generator().manual_seed(5)) if rank == 0 else None
    res["route"] = R.route_rows(xr, [0], list(range(1, world)), 12, "unit_norm", 2.0)
    # sharded BatchTopK: a coarse value grid makes ties at the threshold certain
    hg = torch.Generator().manual_seed(3)
    H = (torch.randint(-6, 10, (16, 12 * world), generator=hg).float() * 0.25)
    res["btk"] = R.sharded_batch_topk(H[:, rank * 12 : (rank + 1) * 12].contiguous(), 2.5, 8)
    # FSDP reduce-scatter: rank-mean of every rank's gradient rows, sharded by latent owner
    gr = torch.randn(8 * world, 16, generator=torch.Generator().manual_seed(40 + rank))
    res["fsdp"] = R.fsdp_reduce_scatter(gr)
    torch.save(res, os.path.join(out_dir, f"r{rank}.pt"))
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_reference_algorithms(tmp_path, world):
    mp.spawn(_worker, args=(world, _port(), str(tmp_path)), nprocs=world, join=True)
    r = [torch.load(tmp_path / f"r{i}.pt") for i in range(world)]
    xs = [torch.randn(10_000, generator=torch.Generator().manual_seed(i)) for i in range(world)]
    want = sum(xs) * 0.5
    for i in range(world):
        assert torch.allclose(r[i]["ar_f32"], want, atol=1e-5)
        assert torch.allclose(r[i]["ar_f32_sq"][0], want[:2048].square().sum(), rtol=1e-5)
        assert torch.equal(r[i]["ar_bf16"], r[0]["ar_bf16"])
    # decode: owner rows of the summed partials + b_dec
    B, D = 6 * world, 8
    total = sum(ri["partial"] for ri in r)
    tgt = torch.randn(B, D, generator=torch.Generator().manual_seed(99))
    Bo = B // world
    for i in range(world):
        xh, loss_row, dx = r[i]["rs"]
        rows = slice(i * Bo, (i + 1) * Bo)
        assert torch.allclose(xh, total[rows] + 1.0, atol=1e-5)
        assert torch.allclose(loss_row, (total[rows] + 1.0 - tgt[rows]).square().sum(-1), rtol=1e-5)
        assert torch.allclose(dx.float(), ((total + 1.0 - tgt) * 2.0 / B).to(torch.bfloat16).float())
    # merge: every rank offers the same candidates; rank s's local id i is global s*10+i, and the
    # global top-3 takes the larger value first, then the smaller global id
    vals = [[5.0, 3.0, 1.0], [2.0, 2.0, 0.5]]
    idx = [[0, 1, 2], [3, 4, -1]]
    for b in range(2):
        pool = sorted((-vals[b][i], s * 10 + idx[b][i], s, i)
                      for s in range(world) for i in range(3) if idx[b][i] >= 0)
        win = {(s, i) for _, _, s, i in pool[:3]}
        for s in range(world):
            assert r[s]["keep"][b].tolist() == [(s, i) in win for i in range(3)]
    assert r[0]["keep"][0].tolist() == [True, world == 2, False]
    # routing: consumers hold the unit-norm rows of their shares, in order
    x = torch.randn(12, 4, generator=torch.Generator().manual_seed(5))
    xn = (x / x.norm(dim=-1, keepdim=True) * 2.0).to(torch.bfloat16)
    got = torch.cat([r[i]["route"] for i in range(1, world)])
    assert torch.equal(got, xn)
    assert r[0]["route"] is None
    # sharded BatchTopK = the top K of the full batch, ties in (row, latent) order
    H = (torch.randint(-6, 10, (16, 12 * world), generator=torch.Generator().manual_seed(3)).float() * 0.25)
    K = round(2.5 * 16)
    flat = H.reshape(-1)
    order = sorted(range(flat.numel()), key=lambda i: (-float(flat[i]), i))  # (row, latent) = flat order
    want = torch.zeros(flat.numel(), dtype=torch.bool)
    for i in order[:K]:
        if flat[i] > 0:
            want[i] = True
    got = torch.cat([r[i]["btk"] for i in range(world)], dim=1).reshape(-1)
    assert int(got.sum()) == K
    assert torch.equal(got, want)
    # FSDP reduce-scatter: the shards concatenate to the bf16-rounded mean of the ranks' rows
    grs = [torch.randn(8 * world, 16, generator=torch.Generator().manual_seed(40 + i)).to(torch.bfloat16).float()
           for i in range(world)]
    mean = (sum(grs) / world).to(torch.bfloat16)
    full = torch.cat([r[i]["fsdp"] for i in range(world)])
    assert full.shape == (8 * world, 16) and torch.allclose(full.float(), mean.float(), atol=1e-2, rtol=1e-2)
