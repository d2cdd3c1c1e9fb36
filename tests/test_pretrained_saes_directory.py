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


def test_shipped_index_holds_the_full_directory():
    from saelens_b200.loading.pretrained_saes_directory import directory_files

    assert any(p.endswith("pretrained_saes_index.json.gz") for p in directory_files())
    d = get_pretrained_saes_directory()
    assert len(d) >= 150
    assert sum(len(v.saes_map) for v in d.values()) > 10_000
    assert len(d["gpt2-small-res-jb"].saes_map) == 13  # every layer's resid_pre, plus the last resid_post
    assert get_repo_id_and_folder_name("gemma-scope-2b-pt-res-canonical", "layer_12/width_16k/canonical") == \
        ("google/gemma-scope-2b-pt-res", "layer_12/width_16k/average_l0_82")
    # A folder name written as a bare number in the source YAML stays a number.
    assert d["mntss-gemma-2-2b-2.5m-clt-as-per-layer"].saes_map["layer_0"] == 0


def _sample_directory():
    return {
        "rel-a": {"repo_id": "org/a", "model": "m", "conversion_func": None,
                  "links": {"model": "https://example.org"},
                  "config_overrides": {"model_from_pretrained_kwargs": {"center_writing_weights": True}},
                  "saes": [{"id": "s0", "path": "s0", "l0": 12.0, "neuronpedia": "m/0"},
                           {"id": "s1", "path": "deep/s1", "variance_explained": 0.7,
                            "norm_scaling_factor": 3.5},
                           {"id": "layer_0", "path": 0}]},
        "rel-b": {"repo_id": "org/b", "model": "m2", "conversion_func": "gemma_2",
                  "saes": [{"id": "x", "path": "y"}]},
    }


def test_index_round_trip_is_lossless():
    from saelens_b200.loading.pretrained_index import compact_directory, expand_index
    from saelens_b200.loading.pretrained_saes_directory import _parse

    data = _sample_directory()
    back = expand_index(compact_directory(data))
    assert back == data
    assert _parse(back) == _parse(data)
    parsed = _parse(back)["rel-a"]
    assert parsed.expected_l0 == {"s0": 12.0, "s1": 0.0, "layer_0": 0.0}
    assert parsed.expected_var_explained["s1"] == 0.7 and parsed.expected_var_explained["s0"] == 1.0
    assert parsed.norm_scaling_factor == {"s1": 3.5}


def test_build_index_from_yaml_and_extra_index_file(tmp_path, monkeypatch):
    import yaml

    from saelens_b200.loading import pretrained_saes_directory as psd
    from saelens_b200.loading.pretrained_index import build_index, load_index

    data = _sample_directory()
    src = tmp_path / "dir.yaml"
    src.write_text(yaml.safe_dump(data))
    out = tmp_path / "extra.json.gz"
    assert build_index(str(src), str(out)) == 2
    first = out.read_bytes()
    build_index(str(src), str(out))
    assert out.read_bytes() == first  # deterministic output
    assert psd._parse(load_index(str(out))) == psd._parse(data)
    monkeypatch.setenv("SAELENS_B200_PRETRAINED_YAML", str(out))
    psd._load_files.cache_clear()
    try:
        assert get_repo_id_and_folder_name("rel-b", "x") == ("org/b", "y")
        assert get_conversion_loader_name("rel-b") == "gemma_2"
    finally:
        monkeypatch.delenv("SAELENS_B200_PRETRAINED_YAML")
        psd._load_files.cache_clear()
