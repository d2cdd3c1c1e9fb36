"""Compact, columnar index of the pretrained SAE directory.

The directory of published SAE releases (release -> HF repo, per-SAE folder, expected L0 and
variance explained, Neuronpedia id, norm scaling factor) is public metadata that must match the
Hugging Face repositories exactly, so its entries are the reference's (sae_lens/
pretrained_saes.yaml, 156 releases, 13k SAEs; schema read by sae_lens/loading/
pretrained_saes_directory.py:23-59).  As a 1.5 MB YAML file it is slow to parse at import (about
10 s with PyYAML's pure-Python loader); the package ships it instead as gzip-compressed JSON in
columns, one object per release:

    {"repo_id", "model", "conversion_func", "config_overrides", "links",
     "ids": [...], "paths": [path, or null where the path equals the id],
     "l0": [float or null], "neuronpedia": [str or null],
     "variance_explained": {position: float}, "norm_scaling_factor": {position: float}}

`expand_index` turns that back into the YAML schema's dict (absent fields stay absent, so the
defaults of the directory parser apply unchanged).  `build_index` makes the file from any YAML in
the directory schema:

    python -m saelens_b200.loading.pretrained_index <pretrained_saes.yaml> [out.json.gz]
"""

from __future__ import annotations

import gzip
import json
import os
import sys
from typing import Any

INDEX_NAME = "pretrained_saes_index.json.gz"


def compact_directory(data: dict[str, Any]) -> dict[str, Any]:
    """YAML-schema directory dict -> columnar dict (lossless for the fields the parser reads)."""
    out: dict[str, Any] = {}
    for release, value in data.items():
        if "saes" not in value:
            raise KeyError(f"Missing 'saes' key in {release}")
        saes = value["saes"]
        entry: dict[str, Any] = {k: value[k] for k in ("repo_id", "model") if k in value}
        for k in ("conversion_func", "config_overrides", "links"):
            if value.get(k) is not None:
                entry[k] = value[k]
        entry["ids"] = [s["id"] for s in saes]
        entry["paths"] = [None if s["path"] == s["id"] else s["path"] for s in saes]
        for col in ("l0", "neuronpedia"):
            vals = [s.get(col) for s in saes]
            if any(v is not None for v in vals):
                entry[col] = vals
        for col in ("variance_explained", "norm_scaling_factor"):
            sparse = {str(i): s[col] for i, s in enumerate(saes) if col in s}
            if sparse:
                entry[col] = sparse
        out[release] = entry
    return out


def expand_index(index: dict[str, Any]) -> dict[str, Any]:
    """Columnar dict -> YAML-schema directory dict."""
    out: dict[str, Any] = {}
    for release, entry in index.items():
        ids, paths = entry["ids"], entry["paths"]
        if len(ids) != len(paths):
            raise ValueError(f"{release}: {len(ids)} ids but {len(paths)} paths")
        saes: list[dict[str, Any]] = []
        for i, sid in enumerate(ids):
            info: dict[str, Any] = {"id": sid, "path": sid if paths[i] is None else paths[i]}
            for col in ("l0", "neuronpedia"):
                if col in entry and entry[col][i] is not None:
                    info[col] = entry[col][i]
            for col in ("variance_explained", "norm_scaling_factor"):
                v = entry.get(col, {}).get(str(i))
                if v is not None:
                    info[col] = v
            saes.append(info)
        value: dict[str, Any] = {k: entry[k] for k in ("repo_id", "model") if k in entry}
        value["conversion_func"] = entry.get("conversion_func")
        for k in ("config_overrides", "links"):
            if k in entry:
                value[k] = entry[k]
        value["saes"] = saes
        out[release] = value
    return out


def load_index(path: str) -> dict[str, Any]:
    """Read a columnar index file and return the YAML-schema directory dict."""
    with gzip.open(path, "rt", encoding="utf-8") as f:
        return expand_index(json.load(f))


def build_index(yaml_path: str, out_path: str) -> int:
    """Write the columnar index of a directory YAML; returns the number of releases."""
    import yaml

    with open(yaml_path) as f:
        data = yaml.load(f, Loader=getattr(yaml, "CSafeLoader", yaml.SafeLoader))
    index = compact_directory(data)
    # mtime=0 keeps the file byte-identical across rebuilds of the same YAML.
    with open(out_path, "wb") as raw, gzip.GzipFile(fileobj=raw, mode="wb", mtime=0) as gz:
        gz.write(json.dumps(index, separators=(",", ":"), sort_keys=False).encode("utf-8"))
    return len(index)


def main(argv: list[str] | None = None) -> None:
    argv = sys.argv[1:] if argv is None else argv
    if not argv:
        raise SystemExit("usage: python -m saelens_b200.loading.pretrained_index <yaml> [out.json.gz]")
    out = argv[1] if len(argv) > 1 else os.path.join(os.path.dirname(os.path.abspath(__file__)), INDEX_NAME)
    n = build_index(argv[0], out)
    print(f"wrote {n} releases to {out} ({os.path.getsize(out)} bytes)")


if __name__ == "__main__":
    main()
