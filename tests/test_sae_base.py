"""SAE base behaviour for every training architecture: config round trips, metadata, activation-norm
folding, checkpoint save / load, memory-lean disk loading and pretrained loading with norm folding
(behaviour of sae_lens/saes/sae.py; cases follow tests/saes/test_sae.py)."""

import copy
import pickle
import tracemalloc
from typing import Any
from unittest import mock

import pytest
import torch

from saelens_b200.models.sae import SAE, SAEConfig, SAEMetadata, TrainingSAE, TrainingSAEConfig
from saelens_b200.registry import get_sae_class, get_sae_training_class

ARCHS = ["standard", "gated", "topk", "jumprelu", "batchtopk", "matryoshka_batchtopk"]


def _cfg(arch: str, d_in: int = 16, d_sae: int = 32) -> TrainingSAEConfig:
    extra: dict[str, Any] = {}
    if arch in ("topk", "batchtopk", "matryoshka_batchtopk"):
        extra["k"] = 4
    if arch == "matryoshka_batchtopk":
        extra["matryoshka_widths"] = [8, d_sae]
    return get_sae_training_class(arch)[1](d_in=d_in, d_sae=d_sae, **extra)


def _random_params(sae: torch.nn.Module) -> None:
    torch.manual_seed(0)
    with torch.no_grad():
        for p in sae.parameters():
            p.copy_(torch.randn_like(p) * 0.3)


@pytest.mark.parametrize("arch", ARCHS)
def test_training_config_dict_roundtrip(arch):
    cfg = _cfg(arch)
    back = TrainingSAEConfig.from_dict(cfg.to_dict())
    assert back.to_dict() == cfg.to_dict()
    assert type(back) is type(cfg) is get_sae_training_class(arch)[1]


@pytest.mark.parametrize("arch", ARCHS)
def test_inference_config_dict_roundtrip(arch):
    d = _cfg(arch).get_inference_sae_cfg_dict()
    back = SAEConfig.from_dict(d)
    want = "jumprelu" if arch in ("batchtopk", "matryoshka_batchtopk") else arch
    assert back.architecture() == want
    assert back.to_dict() == d
    assert type(back) is get_sae_class(want)[1]


def test_metadata_behaves_like_a_dict_with_none_default():
    m = SAEMetadata(model_name="m", hook_name="h", custom_field="v")
    assert (m.model_name, m.hook_name, m.custom_field) == ("m", "h", "v")
    assert m.nonexistent is None and m["nonexistent"] is None
    m["k"] = 42
    m.dyn = "x"
    assert m["k"] == 42 and "k" in m and "dyn" in m and "missing" not in m
    assert m.get("missing") is None and m.get("missing", "d") == "d" and m.get("k") == 42
    assert {"model_name", "hook_name", "custom_field", "k", "dyn", "sae_lens_version",
            "sae_lens_training_version"} <= set(m.keys())
    assert ("k", 42) in set(m.items()) and 42 in list(m.values())
    assert "SAEMetadata" in repr(m) and "custom_field" in repr(m)


def test_metadata_roundtrip_equality_copy_pickle():
    m = SAEMetadata(model_name="test", hook_name="hook", custom=123, nested={"key": "value"})
    back = SAEMetadata.from_dict(m.to_dict())
    assert back == m and back.custom == 123
    assert SAEMetadata(a=1) != SAEMetadata(a=2) and SAEMetadata(a=1) != "not metadata"
    c = copy.deepcopy(m)
    assert c == m and c is not m and c.nested is not m.nested
    assert pickle.loads(pickle.dumps(m)) == m


def test_metadata_versions():
    m = SAEMetadata()
    assert m.sae_lens_version and m.sae_lens_training_version
    assert SAEMetadata(sae_lens_version="custom").sae_lens_version == "custom"


def test_deprecated_tuple_access():
    sae = SAE.from_dict(_cfg("standard").get_inference_sae_cfg_dict())
    with pytest.warns(DeprecationWarning, match="Unpacking SAE objects is deprecated"):
        s, d, sp = sae
    assert s is sae and d == sae.cfg.to_dict() and sp is None
    with pytest.warns(DeprecationWarning, match="Indexing SAE objects is deprecated"):
        assert sae[0] is sae
    with pytest.warns(DeprecationWarning, match="Getting length of SAE objects is deprecated"):
        assert len(sae) == 3


@pytest.mark.parametrize("arch", ARCHS)
def test_fold_activation_norm_scaling_factor(arch):
    sae = TrainingSAE.from_dict(_cfg(arch).to_dict())
    _random_params(sae)
    x = torch.randn(100, 16)
    with torch.no_grad():
        out0, f0 = sae(x), sae.encode(x)
        sae.fold_activation_norm_scaling_factor(2.0)
        out1, f1 = 2.0 * sae(x / 2.0), sae.encode(x / 2.0)
    torch.testing.assert_close(out1, out0, atol=1e-4, rtol=1e-4)
    if arch in ("topk", "batchtopk", "matryoshka_batchtopk"):
        # decoder-norm rescaling of the activations folds the factor into the features
        torch.testing.assert_close(f1, f0 / 2.0, atol=1e-4, rtol=1e-4)
    else:
        torch.testing.assert_close(f1, f0, atol=1e-4, rtol=1e-4)


@pytest.mark.parametrize("arch", ARCHS)
def test_training_checkpoint_roundtrip(arch, tmp_path):
    sae = TrainingSAE.from_dict(_cfg(arch).to_dict())
    _random_params(sae)
    sae.save_model(tmp_path)
    other = TrainingSAE.from_dict(_cfg(arch).to_dict())
    other.load_weights_from_checkpoint(tmp_path)
    for (n, a), (_, b) in zip(sae.named_parameters(), other.named_parameters()):
        torch.testing.assert_close(a, b, atol=1e-6, rtol=1e-4, msg=n)


@pytest.mark.parametrize("arch", ["standard", "gated", "topk", "jumprelu"])
def test_load_from_disk_builds_on_meta_and_assigns(arch, tmp_path):
    sae = TrainingSAE.from_dict(_cfg(arch, 64, 256).to_dict())
    _random_params(sae)
    sae.save_model(tmp_path)
    seen = {"meta": False, "assign": False}
    orig = SAE.load_state_dict

    def spy(self, state_dict, strict=True, assign=False):
        seen["meta"] |= any(p.device.type == "meta" for p in self.parameters())
        seen["assign"] |= assign
        return orig(self, state_dict, strict=strict, assign=assign)

    with mock.patch.object(SAE, "load_state_dict", spy):
        loaded = SAE.load_from_disk(tmp_path, device="cpu")
    assert seen == {"meta": True, "assign": True}
    assert loaded.W_enc.device.type == "cpu"


def test_load_from_disk_peak_memory_below_two_copies(tmp_path):
    d_in, d_sae = 512, 4096
    sae = TrainingSAE.from_dict(_cfg("standard", d_in, d_sae).to_dict())
    _random_params(sae)
    sae.save_model(tmp_path)
    param_bytes = (2 * d_in * d_sae + d_sae + d_in) * 4
    tracemalloc.start()
    tracemalloc.reset_peak()
    loaded = SAE.load_from_disk(tmp_path, device="cpu")
    _, peak = tracemalloc.get_traced_memory()
    tracemalloc.stop()
    assert loaded is not None and peak < 1.5 * param_bytes


def test_from_pretrained_folds_norm_scaling_factor(tmp_path):
    from saelens_b200.loading import pretrained_sae_loaders as L
    from saelens_b200.loading import pretrained_saes_directory as D

    sae = TrainingSAE.from_dict(_cfg("standard", 32, 64).to_dict())
    _random_params(sae)
    sae.save_model(tmp_path)
    cfg_dict, state = L.sae_lens_disk_loader(tmp_path, device="cpu")
    cfg_dict["normalize_activations"] = "expected_average_only_in"
    W_enc, W_dec, b_dec = state["W_enc"].clone(), state["W_dec"].clone(), state["b_dec"].clone()

    def loader(repo_id, folder_name, device="cpu", force_download=False, cfg_overrides=None):
        return dict(cfg_dict), dict(state), None

    info = type("Info", (), {"conversion_func": None, "saes_map": {"sid": {}}})()
    with mock.patch.dict(L.NAMED_PRETRAINED_SAE_LOADERS, {"mock_loader": loader}), \
         mock.patch.object(D, "get_pretrained_saes_directory", return_value={"rel": info}), \
         mock.patch.object(D, "get_conversion_loader_name", return_value="mock_loader"), \
         mock.patch.object(D, "get_repo_id_and_folder_name", return_value=("org/repo", "f")), \
         mock.patch.object(D, "get_config_overrides", return_value={}), \
         mock.patch.object(D, "get_norm_scaling_factor", return_value=2.0):
        loaded = SAE.from_pretrained("rel", "sid", device="cpu")
    torch.testing.assert_close(loaded.W_enc, W_enc * 2.0)
    torch.testing.assert_close(loaded.W_dec, W_dec / 2.0)
    torch.testing.assert_close(loaded.b_dec, b_dec / 2.0)
    assert loaded.cfg.normalize_activations == "none"


def test_from_pretrained_unknown_release_and_id():
    with pytest.raises(ValueError, match="not found in pretrained SAEs directory"):
        SAE.from_pretrained("no-such-release", "x")
