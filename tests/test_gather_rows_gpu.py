"""Native two-source row gather (ops/csrc/rows.cu) and the mixing buffer's shuffle on CUDA, against
`torch.cat(...)[perm]` and the CPU path of the same buffer."""

from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():
    pytest.skip("needs a CUDA device", allow_module_level=True)

from saelens_b200 import ops  # noqa: E402
from saelens_b200.training.mixing_buffer import mixing_buffer  # noqa: E402


@pytest.mark.parametrize("dtype,shape", [(torch.bfloat16, (4096,)), (torch.float32, (768,)), (torch.float32, (5,)),
                                         (torch.float16, (3, 6)), (torch.bfloat16, (7,))])
def test_gather_matches_cat_then_index(dtype, shape) -> None:
    g = torch.Generator().manual_seed(0)
    a = torch.randn(1000, *shape, generator=g).to(dtype).cuda()
    b = torch.randn(333, *shape, generator=g).to(dtype).cuda()
    perm = torch.randperm(1333, generator=g).cuda()
    got = ops.gather_rows(a, b, perm)
    assert torch.equal(got, torch.cat([a, b])[perm])
    assert torch.equal(ops.gather_rows(a, None, perm[perm < 1000]), a[perm[perm < 1000]])


def test_gather_from_strided_views_and_out_of_range_rows() -> None:
    base = torch.randn(64, 2, 32, device="cuda")
    a = base[:, 0]  # rows 256 bytes apart, each 128 contiguous bytes
    b = base[:10, 1]
    perm = torch.tensor([3, 70, 1, 64, 999, -1, 5], device="cuda")
    out = torch.full((7, 32), 7.0, device="cuda")
    bad = torch.zeros(1, dtype=torch.int32, device="cuda")
    ops.native().gather_rows(a, b, perm, out, bad)
    src = torch.cat([a, b])
    for i, p in enumerate(perm.tolist()):
        if 0 <= p < 74:
            assert torch.equal(out[i], src[p])
        else:
            assert bool((out[i] == 7.0).all())
    assert int(bad) == 2


@pytest.mark.parametrize("mix", [0.0, 0.5, 1.0])
def test_mixing_buffer_on_cuda_serves_the_cpu_stream(mix) -> None:
    g = torch.Generator().manual_seed(1)
    batches = [torch.randn(100, 16, generator=g) for _ in range(23)]

    def run(dev):
        gen = torch.Generator().manual_seed(5)
        return [t.cpu() for t in mixing_buffer(400, 64, iter([b.to(dev) for b in batches]), mix, gen)]

    cpu, gpu = run("cpu"), run("cuda")
    assert len(cpu) == len(gpu)
    for x, y in zip(cpu, gpu):
        assert torch.equal(x, y)


def test_mixing_buffer_dict_batches_on_cuda() -> None:
    g = torch.Generator().manual_seed(2)
    batches = [{"a": torch.randn(50, 8, generator=g), "b": torch.randn(50, 4, generator=g).bfloat16()}
               for _ in range(10)]

    def run(dev):
        gen = torch.Generator().manual_seed(9)
        src = iter([{k: v.to(dev) for k, v in b.items()} for b in batches])
        return [{k: v.cpu() for k, v in t.items()} for t in mixing_buffer(200, 32, src, 0.5, gen)]

    for x, y in zip(run("cpu"), run("cuda"), strict=True):
        assert torch.equal(x["a"], y["a"]) and torch.equal(x["b"], y["b"])
