"""Small helpers shared across the package (dtype names, dataclass filtering, temp dirs)."""

from __future__ import annotations

import dataclasses
import tempfile
from collections.abc import Iterator
from contextlib import contextmanager
from pathlib import Path
from typing import Any

import torch

DTYPE_MAP: dict[str, torch.dtype] = {
    "float32": torch.float32,
    "float64": torch.float64,
    "float16": torch.float16,
    "bfloat16": torch.bfloat16,
    "torch.float32": torch.float32,
    "torch.float64": torch.float64,
    "torch.float16": torch.float16,
    "torch.bfloat16": torch.bfloat16,
    "fp32": torch.float32,
    "fp16": torch.float16,
    "bf16": torch.bfloat16,
}


def str_to_dtype(dtype: str | torch.dtype) -> torch.dtype:
    if isinstance(dtype, torch.dtype):
        return dtype
    try:
        return DTYPE_MAP[dtype]
    except KeyError as e:
        raise ValueError(f"Invalid dtype: {dtype!r}; expected one of {sorted(DTYPE_MAP)}") from e


def dtype_to_str(dtype: torch.dtype | str) -> str:
    if isinstance(dtype, str):
        return dtype_to_str(str_to_dtype(dtype))
    for name in ("float32", "float64", "float16", "bfloat16"):
        if DTYPE_MAP[name] == dtype:
            return name
    raise ValueError(f"Invalid dtype: {dtype}")


def filter_valid_dataclass_fields(data: dict[str, Any] | Any, cls: Any,
                                  whitelist_fields: list[str] | None = None) -> dict[str, Any]:
    """The entries of `data` (a dict or a dataclass instance) that are init fields of dataclass
    `cls`, plus any `whitelist_fields` present in `data`."""
    if not dataclasses.is_dataclass(cls):
        raise ValueError(f"{cls} is not a dataclass")
    if dataclasses.is_dataclass(data) and not isinstance(data, type):
        data = {f.name: getattr(data, f.name) for f in dataclasses.fields(data)}
    elif not isinstance(data, dict):
        raise ValueError(f"{data!r} is not a dict or dataclass")
    names = {f.name for f in dataclasses.fields(cls) if f.init}
    if whitelist_fields:
        names |= set(whitelist_fields)
    return {k: v for k, v in data.items() if k in names}


@contextmanager
def path_or_tmp_dir(path: str | Path | None) -> Iterator[Path]:
    if path is None:
        with tempfile.TemporaryDirectory() as d:
            yield Path(d)
    else:
        yield Path(path)


def get_special_token_ids(tokenizer: Any) -> list[int]:
    ids: set[int] = set()
    for attr in ("bos_token_id", "eos_token_id", "pad_token_id", "unk_token_id", "sep_token_id"):
        v = getattr(tokenizer, attr, None)
        if v is not None:
            ids.add(int(v))
    extra = getattr(tokenizer, "all_special_ids", None)
    if extra:
        ids.update(int(i) for i in extra)
    return sorted(ids)


def extract_stop_at_layer_from_hook_name(hook_name: str) -> int | None:
    """`blocks.6.hook_resid_pre` -> 7: the LM forward can stop after the hook's layer."""
    parts = hook_name.split(".")
    for i, p in enumerate(parts):
        if p == "blocks" and i + 1 < len(parts) and parts[i + 1].isdigit():
            return int(parts[i + 1]) + 1
    return None


def extract_layer_from_tlens_hook_name(hook_name: str) -> int | None:
    """The layer index of a TransformerLens-style hook name (`blocks.6.hook_resid_pre` -> 6): the
    first dot-delimited all-digit component, or None."""
    for part in hook_name.split(".")[1:-1]:
        if part.isdigit():
            return int(part)
    return None


def extract_stop_at_layer_from_tlens_hook_name(hook_name: str) -> int | None:
    """The `stop_at_layer` that still runs the hook's layer (layer + 1), or None."""
    layer = extract_layer_from_tlens_hook_name(hook_name)
    return None if layer is None else layer + 1


@contextmanager
def temporary_seed(seed: int | None) -> Iterator[None]:
    """Seed torch's global RNG inside the block only (CPU and CUDA states are restored after);
    `None` leaves the RNG alone."""
    if seed is None:
        yield
        return
    with torch.random.fork_rng():
        torch.manual_seed(seed)
        yield


def cosine_similarities(a: torch.Tensor, b: torch.Tensor | None = None) -> torch.Tensor:
    """Pairwise cosine similarities between the rows of a [n, d] and b [m, d] (b defaults to a)."""
    a_n = a / a.norm(dim=-1, keepdim=True).clamp(min=1e-12)
    b_n = a_n if b is None else b / b.norm(dim=-1, keepdim=True).clamp(min=1e-12)
    return a_n @ b_n.T
