"""Directory of pretrained SAE releases (release -> HF repo, per-SAE folders and metadata).

Same YAML schema as the reference's directory (sae_lens/loading/pretrained_saes_directory.py:
release keys with `repo_id`, `model`, `conversion_func`, `saes: [{id, path, l0,
variance_explained, neuronpedia, norm_scaling_factor}]`, `config_overrides`).  The package ships
the full directory of published releases (156 releases, 13k SAEs) as a gzip-compressed columnar
index (`pretrained_saes_index.json.gz`, read by `pretrained_index.load_index` in about 0.1 s).
Sources, in this order of precedence (later entries override earlier ones):
1. the shipped `pretrained_saes.yaml` (a few hand-kept releases);
2. the shipped index;
3. the `pretrained_saes.yaml` of an installed `sae_lens` package, located on `sys.path` without
   importing it (same schema; a newer package brings newer releases);
4. every file named in `SAELENS_B200_PRETRAINED_YAML` (`os.pathsep`-separated; a `.json.gz`
   name is read as an index);
5. releases added at runtime with `register_release`.
"""

from __future__ import annotations

import os
from dataclasses import dataclass
from functools import cache
from importlib.resources import files
from typing import Any

import yaml

from .pretrained_index import INDEX_NAME, load_index


@dataclass
class PretrainedSAELookup:
    release: str
    repo_id: str
    model: str
    conversion_func: str | None
    saes_map: dict[str, str]
    expected_var_explained: dict[str, float]
    expected_l0: dict[str, float]
    neuronpedia_id: dict[str, str | None]
    norm_scaling_factor: dict[str, float]
    config_overrides: dict[str, Any] | None


_EXTRA: dict[str, PretrainedSAELookup] = {}


def _parse(data: dict[str, Any]) -> dict[str, PretrainedSAELookup]:
    out: dict[str, PretrainedSAELookup] = {}
    for release, value in (data or {}).items():
        if "saes" not in value:
            raise KeyError(f"Missing 'saes' key in {release}")
        saes, ve, l0, npd, nsf = {}, {}, {}, {}, {}
        for info in value["saes"]:
            sid = info["id"]
            saes[sid] = info["path"]
            ve[sid] = info.get("variance_explained", 1.0)
            l0[sid] = info.get("l0", 0.0)
            npd[sid] = info.get("neuronpedia")
            if "norm_scaling_factor" in info:
                nsf[sid] = info["norm_scaling_factor"]
        out[release] = PretrainedSAELookup(
            release=release, repo_id=value["repo_id"], model=value["model"],
            conversion_func=value.get("conversion_func"), saes_map=saes, expected_var_explained=ve,
            expected_l0=l0, neuronpedia_id=npd, norm_scaling_factor=nsf,
            config_overrides=value.get("config_overrides"),
        )
    return out


def installed_sae_lens_directory() -> str | None:
    """Path of an installed `sae_lens` package's pretrained_saes.yaml, found without importing it."""
    import importlib.util

    try:
        spec = importlib.util.find_spec("sae_lens")
    except (ImportError, ValueError):
        return None
    if spec is None or not spec.submodule_search_locations:
        return None
    for root in spec.submodule_search_locations:
        path = os.path.join(root, "pretrained_saes.yaml")
        if os.path.isfile(path):
            return path
    return None


def directory_files() -> list[str]:
    """The YAML files the directory is read from, lowest precedence first."""
    here = files("saelens_b200.loading")
    out = [str(here.joinpath("pretrained_saes.yaml"))]
    index = str(here.joinpath(INDEX_NAME))
    if os.path.isfile(index):
        out.append(index)
    ref = installed_sae_lens_directory()
    if ref:
        out.append(ref)
    for extra in os.environ.get("SAELENS_B200_PRETRAINED_YAML", "").split(os.pathsep):
        if extra and os.path.exists(extra):
            out.append(extra)
    return out


@cache
def _load_files() -> dict[str, PretrainedSAELookup]:
    directory: dict[str, PretrainedSAELookup] = {}
    for path in directory_files():
        if path.endswith(".json.gz"):
            directory.update(_parse(load_index(path)))
            continue
        with open(path) as f:
            directory.update(_parse(yaml.load(f, Loader=getattr(yaml, "CSafeLoader", yaml.SafeLoader))))
    return directory


def get_pretrained_saes_directory() -> dict[str, PretrainedSAELookup]:
    return {**_load_files(), **_EXTRA}


def register_release(release: str, entry: dict[str, Any]) -> None:
    """Add a release at runtime (same schema as one YAML entry)."""
    _EXTRA.update(_parse({release: entry}))


def get_norm_scaling_factor(release: str, sae_id: str) -> float | None:
    info = get_pretrained_saes_directory().get(release)
    return None if info is None else info.norm_scaling_factor.get(sae_id)


def get_repo_id_and_folder_name(release: str, sae_id: str) -> tuple[str, str]:
    info = get_pretrained_saes_directory().get(release)
    if info is None:
        return release, sae_id
    if sae_id not in info.saes_map:
        raise ValueError(f"SAE ID '{sae_id}' not found in release '{release}'")
    return info.repo_id, info.saes_map[sae_id]


def get_config_overrides(release: str, sae_id: str) -> dict[str, Any]:
    info = get_pretrained_saes_directory().get(release)
    out: dict[str, Any] = {}
    if info is not None:
        out = {**(info.config_overrides or {})}
        if sae_id in info.neuronpedia_id:
            out["neuronpedia_id"] = info.neuronpedia_id[sae_id]
    return out


def get_conversion_loader_name(release: str) -> str:
    info = get_pretrained_saes_directory().get(release)
    if info is not None and info.conversion_func is not None:
        return info.conversion_func
    return "sae_lens"


def get_releases_for_repo_id(repo_id: str) -> list[str]:
    return [r for r, v in get_pretrained_saes_directory().items() if v.repo_id == repo_id]
