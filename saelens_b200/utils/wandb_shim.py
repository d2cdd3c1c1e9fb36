"""Weights & Biases access.  Uses `wandb` when it is installed; otherwise every call is recorded
to `$SAELENS_B200_WANDB_DIR/wandb_log.jsonl` (default: ./wandb_offline) so training with
`log_to_wandb=True` still works offline."""

from __future__ import annotations

import json
import os
import time
from typing import Any

import importlib.util

AVAILABLE = importlib.util.find_spec("wandb") is not None
_wandb: Any = None  # imported on first use (importing wandb takes seconds)


def _module() -> Any:
    global _wandb
    if _wandb is None and AVAILABLE:
        try:  # pragma: no cover - depends on the environment
            import wandb  # type: ignore[import-not-found]

            _wandb = wandb
        except Exception:  # noqa: BLE001
            return None
    return _wandb


def _live() -> bool:
    """True when a real wandb run is active; otherwise calls go to the offline JSONL log."""
    m = _module() if "wandb" in __import__("sys").modules else None
    return m is not None and getattr(m, "run", None) is not None


def _log_path() -> str:
    d = os.environ.get("SAELENS_B200_WANDB_DIR", "wandb_offline")
    os.makedirs(d, exist_ok=True)
    return os.path.join(d, "wandb_log.jsonl")


def _jsonable(v: Any) -> Any:
    try:
        import numpy as np
        import torch

        if isinstance(v, torch.Tensor):
            return v.detach().float().cpu().tolist() if v.numel() > 1 else float(v.item())
        if isinstance(v, np.ndarray):
            return {"histogram_of": int(v.size), "mean": float(v.mean()) if v.size else 0.0}
    except Exception:  # noqa: BLE001
        pass
    if isinstance(v, Histogram):
        return v.summary
    return v if isinstance(v, (int, float, str, bool, type(None), list, dict)) else repr(v)


class Histogram:
    def __init__(self, values: Any):
        import numpy as np

        self._values = values

        arr = np.asarray(values, dtype=float)
        self.summary = {"n": int(arr.size), "mean": float(arr.mean()) if arr.size else 0.0,
                        "min": float(arr.min()) if arr.size else 0.0, "max": float(arr.max()) if arr.size else 0.0}


class Artifact:
    def __init__(self, name: str, type: str, metadata: dict[str, Any] | None = None):  # noqa: A002
        self.name, self.type, self.metadata, self.files = name, type, metadata or {}, []

    def add_file(self, path: str) -> None:
        self.files.append(path)


def init(**kwargs: Any) -> Any:
    m = _module()
    if m is not None:
        return m.init(**kwargs)
    with open(_log_path(), "a") as f:
        f.write(json.dumps({"event": "init", "time": time.time(), **{k: _jsonable(v) for k, v in kwargs.items()}}) + "\n")
    return None


def log(data: dict[str, Any], step: int | None = None) -> None:
    if _live():
        _wandb.log(data, step=step)
        return
    with open(_log_path(), "a") as f:
        f.write(json.dumps({"event": "log", "step": step, **{k: _jsonable(v) for k, v in data.items()}}) + "\n")


def log_artifact(art: Artifact, aliases: list[str] | None = None) -> None:
    if _live():
        a = _wandb.Artifact(art.name, type=art.type, metadata=art.metadata)
        for p in art.files:
            a.add_file(p)
        _wandb.log_artifact(a, aliases=aliases)
        return
    with open(_log_path(), "a") as f:
        f.write(json.dumps({"event": "artifact", "name": art.name, "type": art.type, "files": art.files,
                            "aliases": aliases}) + "\n")


def finish() -> None:
    if _live():
        _wandb.finish()
