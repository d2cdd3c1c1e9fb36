"""Host-side parts of the P2P DDP hook: bucket bound, support check and config default."""

import torch

from saelens_b200.parallel.p2p_ddp_hook import max_bucket_bytes, p2p_hook_supported


def test_reserved_bucket_bytes():
    # small models: the whole gradient (DDP may use a single bucket)
    assert max_bucket_bytes([10, 4 << 20], 1.0) == (4 << 20) + 10
    # large models: cap + largest parameter, at least 256 MiB
    big = [1 << 30, 1 << 30, 1 << 20]
    assert max_bucket_bytes(big, 25.0) == (25 << 20) + (1 << 30)
    assert max_bucket_bytes([200 << 20, 200 << 20], 1.0) == 256 << 20


def test_hook_unsupported_for_cpu_parameters():
    assert not p2p_hook_supported(torch.nn.Linear(4, 4), None)


def test_runner_config_ddp_exchange_default():
    from saelens_b200.config import LanguageModelSAERunnerConfig
    from saelens_b200.models.standard import StandardTrainingSAEConfig

    cfg = LanguageModelSAERunnerConfig(sae=StandardTrainingSAEConfig(d_in=8, d_sae=16), device="cpu")
    assert cfg.ddp_exchange == "nccl"
