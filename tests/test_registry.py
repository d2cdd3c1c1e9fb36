"""Architecture registry (interface of sae_lens/registry.py; cases follow tests/test_registry.py)."""

import pytest

from saelens_b200.registry import (
    get_sae_class,
    get_sae_training_class,
    register_sae_class,
    register_sae_training_class,
)

INFERENCE = ["standard", "gated", "topk", "jumprelu", "transcoder", "skip_transcoder", "jumprelu_transcoder",
             "jumprelu_skip_transcoder", "matching_pursuit", "temporal"]
TRAINING = ["standard", "gated", "topk", "jumprelu", "batchtopk", "matryoshka_batchtopk", "matching_pursuit"]


@pytest.mark.parametrize("arch", INFERENCE)
def test_builtin_inference_architectures(arch):
    cls, cfg_cls = get_sae_class(arch)
    assert cfg_cls.architecture() == arch


@pytest.mark.parametrize("arch", ["batchtopk", "matryoshka_batchtopk"])
def test_batchtopk_family_is_training_only(arch):
    # their inference form is saved as JumpReLU (the learned threshold)
    with pytest.raises(ValueError):
        get_sae_class(arch)


@pytest.mark.parametrize("arch", TRAINING)
def test_builtin_training_architectures(arch):
    cls, cfg_cls = get_sae_training_class(arch)
    assert cfg_cls.architecture() == arch


def test_duplicate_registration_raises():
    cls, cfg_cls = get_sae_class("standard")
    with pytest.raises(ValueError, match="already registered"):
        register_sae_class("standard", cls, cfg_cls)
    tcls, tcfg = get_sae_training_class("standard")
    with pytest.raises(ValueError, match="already registered"):
        register_sae_training_class("standard", tcls, tcfg)


def test_unknown_architecture_raises():
    with pytest.raises(ValueError, match="unknown"):
        get_sae_class("no-such-arch")
    with pytest.raises(ValueError, match="unknown"):
        get_sae_training_class("no-such-arch")
