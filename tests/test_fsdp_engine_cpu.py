"""Host-side part of the sharded data-parallel engine: contiguous latent shards of the module."""

import pytest
import torch

from saelens_b200.models.topk import TopKTrainingSAE, TopKTrainingSAEConfig
from saelens_b200.parallel.fsdp_engine import _shard_module


@pytest.mark.parametrize("world", [2, 4])
def test_shard_module_takes_contiguous_latent_blocks(world):
    torch.manual_seed(0)
    full = TopKTrainingSAE(TopKTrainingSAEConfig(d_in=16, d_sae=64, k=4, device="cpu"))
    for r in range(world):
        sae = TopKTrainingSAE(TopKTrainingSAEConfig(d_in=16, d_sae=64, k=4, device="cpu"))
        sae.load_state_dict(full.state_dict())
        assert _shard_module(sae, r, world) == 64
        n = 64 // world
        assert torch.equal(sae.W_dec, full.W_dec[r * n : (r + 1) * n])
        assert torch.equal(sae.W_enc, full.W_enc[:, r * n : (r + 1) * n])
        assert torch.equal(sae.b_enc, full.b_enc[r * n : (r + 1) * n])
        assert torch.equal(sae.b_dec, full.b_dec)


def test_shard_module_rejects_uneven_split():
    sae = TopKTrainingSAE(TopKTrainingSAEConfig(d_in=16, d_sae=64, k=4, device="cpu"))
    with pytest.raises(ValueError):
        _shard_module(sae, 0, 3)
