"""Pretrained SAE directory lookups (interface of sae_lens/loading/pretrained_saes_directory.py;
cases follow tests/loading/test_pretrained_saes_directory.py, on the releases shipped in-tree and
on a release registered at runtime)."""

import pytest

from saelens_b200.loading.pretrained_saes_directory import (
    get_config_overrides,
    get_conversion_loader_name,
    get_norm_scaling_factor,
    get_pretrained_saes_directory,
    get_releases_for_repo_id,
    get_repo_id_and_folder_name,
    register_release,
)


@pytest.fixture(scope="module", autouse=True)
def scaled_release():
    register_release("test-scaled-release", {
        "repo_id": "org/scaled-saes", "model": "m", "conversion_func": "llama_scope",
        "saes": [{"id": "l0", "path": "L0", "neuronpedia": "m/0-x", "norm_scaling_factor": 112.5,
                  "variance_explained": 0.8, "l0": 30.0}]})


def test_directory_has_shipped_releases():
    d = get_pretrained_saes_directory()
    assert "gpt2-small-res-jb" in d
    info = d["gpt2-small-res-jb"]
    assert info.repo_id == "jbloom/GPT2-Small-SAEs-Reformatted"
    assert info.saes_map["blocks.0.hook_resid_pre"] == "blocks.0.hook_resid_pre"


def test_neuronpedia_ids_are_unique():
    seen = set()
    for info in get_pretrained_saes_directory().values():
        for np_id in info.neuronpedia_id.values():
            if np_id is None:
                continue
            assert np_id not in seen
            seen.add(np_id)


def test_repo_id_and_folder_name():
    assert get_repo_id_and_folder_name("gpt2-small-res-jb", "blocks.0.hook_resid_pre") == \
        ("jbloom/GPT2-Small-SAEs-Reformatted", "blocks.0.hook_resid_pre")
    assert get_repo_id_and_folder_name("release1", "sae1") == ("release1", "sae1")  # a plain hub repo
    with pytest.raises(ValueError):
        get_repo_id_and_folder_name("gpt2-small-res-jb", "sae1")


def test_releases_for_repo_id():
    assert "gpt2-small-res-jb" in get_releases_for_repo_id("jbloom/GPT2-Small-SAEs-Reformatted")
    assert get_releases_for_repo_id("nonexistent/repo") == []


def test_config_overrides():
    o = get_config_overrides("gpt2-small-res-jb", "blocks.0.hook_resid_pre")
    assert o["model_from_pretrained_kwargs"]["center_writing_weights"]
    assert o["neuronpedia_id"] == "gpt2-small/0-res-jb"
    assert get_config_overrides("nonexistent-release", "sae1") == {}


def test_norm_scaling_factor_and_loader_name():
    assert get_norm_scaling_factor("test-scaled-release", "l0") == pytest.approx(112.5)
    assert get_norm_scaling_factor("nonexistent-release", "sae1") is None
    assert get_norm_scaling_factor("gpt2-small-res-jb", "nonexistent-sae") is None
    assert get_norm_scaling_factor("gpt2-small-res-jb", "blocks.0.hook_resid_pre") is None
    assert get_conversion_loader_name("test-scaled-release") == "llama_scope"
    assert get_conversion_loader_name("gpt2-small-res-jb") == "sae_lens"
    info = get_pretrained_saes_directory()["test-scaled-release"]
    assert info.expected_var_explained["l0"] == 0.8 and info.expected_l0["l0"] == 30.0


def test_installed_reference_directory_is_found_without_import(tmp_path, monkeypatch):
    import sys

    from saelens_b200.loading import pretrained_saes_directory as d

    pkg = tmp_path / "sae_lens"
    pkg.mkdir()
    (pkg / "__init__.py").write_text("raise ImportError('must not be imported')\n")
    (pkg / "pretrained_saes.yaml").write_text(
        "ref-release:\n  repo_id: someone/saes\n  model: gpt2\n  conversion_func: null\n"
        "  saes:\n  - id: blocks.0.hook_resid_pre\n    path: blocks.0\n    l0: 12.5\n")
    monkeypatch.syspath_prepend(str(tmp_path))
    monkeypatch.delitem(sys.modules, "sae_lens", raising=False)
    d._load_files.cache_clear()
    try:
        assert d.installed_sae_lens_directory() == str(pkg / "pretrained_saes.yaml")
        got = d.get_pretrained_saes_directory()["ref-release"]
        assert got.repo_id == "someone/saes" and got.expected_l0["blocks.0.hook_resid_pre"] == 12.5
        assert "sae_lens" not in sys.modules
    finally:
        d._load_files.cache_clear()
