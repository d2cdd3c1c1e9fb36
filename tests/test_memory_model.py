"""Memory model: arithmetic on CPU, and the estimate against the measured peak of a native step."""

import pytest
import torch

from saelens_b200.memory_model import MB, estimate


def test_memory_model_components():
    one = estimate(d_in=4096, d_sae=1048576, k=128, batch=16384)
    tp8 = estimate(d_in=4096, d_sae=1048576, k=128, batch=16384, sae_tp=8)
    assert one.sae_state_mb == pytest.approx(8 * tp8.sae_state_mb, rel=1e-3)
    assert tp8.parallel_slabs_mb > 0 and one.parallel_slabs_mb == 0
    # fp32 masters + moments + bf16 copies + bf16 grads = 32 bytes per W element pair
    assert one.sae_state_mb * MB >= 32 * 1048576 * 4096
    dp = estimate(d_in=4096, d_sae=131072, k=64, batch=8192, sae_dp=2)
    assert dp.parallel_slabs_mb * MB == pytest.approx(2 * 131072 * 4096 * 2 * 3)
    prod = estimate(d_in=4096, d_sae=131072, k=64, batch=8192, producer_params=8_000_000_000, producer_tp=2)
    assert prod.producer_mb * MB == pytest.approx(8e9 * 2 / 2)


@pytest.mark.gpu
@pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a GPU")
def test_memory_model_matches_measured_step_peak():
    from saelens_b200.models.topk import TopKTrainingSAE, TopKTrainingSAEConfig
    from saelens_b200.training.engine import FusedTopKEngine

    torch.cuda.empty_cache()
    base = torch.cuda.memory_allocated()
    sae = TopKTrainingSAE(TopKTrainingSAEConfig(d_in=1024, d_sae=65536, k=64, device="cuda"))
    eng = FusedTopKEngine(sae, lr=1e-4)
    x = torch.randn(4096, 1024, device="cuda").to(torch.bfloat16)
    torch.cuda.synchronize()
    torch.cuda.reset_peak_memory_stats()
    eng.step(x)
    torch.cuda.synchronize()
    peak = torch.cuda.max_memory_allocated() - base - x.numel() * 2
    est = estimate(d_in=1024, d_sae=65536, k=64, batch=4096)
    model = (est.sae_state_mb + est.step_buffers_mb) * MB
    assert 0.8 < peak / model < 1.25, (peak / MB, model / MB)


def test_memory_model_sharded_data_parallel_and_slabs():
    kw = dict(d_in=3584, d_sae=131072, k=64, batch=4096)
    ddp = estimate(sae_dp=8, **kw)
    fsdp = estimate(sae_dp=8, fsdp=True, **kw)
    # optimizer state per GPU is an eighth of a replica's; the slab carries the gathered weights
    assert fsdp.sae_state_mb < ddp.sae_state_mb / 4
    N, D = 131072, 3584
    assert fsdp.parallel_slabs_mb * (1 << 20) >= 4 * N * D * 2
    ring = estimate(ring_slots=32, ring_chunk_rows=4096, **kw)
    base = estimate(**kw)
    assert abs((ring.parallel_slabs_mb - base.parallel_slabs_mb) * (1 << 20) - 32 * 4096 * D * 2) < 1
    routed = estimate(route_rows=4096, **kw)
    assert abs((routed.parallel_slabs_mb - base.parallel_slabs_mb) * (1 << 20) - 2 * 4096 * D * 2) < 1
