"""Token sources for the activation pipeline (no hard dependency on HF `datasets`).

`open_token_source(path_or_obj, ...)` returns an iterator of 1-D LongTensor token sequences from:
* an in-memory object: a tensor [n, ctx], a list of token lists / tensors / strings / dicts with
  "tokens" / "input_ids" / "text", or any HF `datasets` object;
* `synthetic:uniform:<vocab>[:<len>]` - uniformly random token ids (for benchmarks);
* a local file or directory: `.jsonl` (one record per line), `.parquet` / `.arrow` (pyarrow),
  `.npy` / `.pt` (token array), or a directory of those;
* anything else is handed to `datasets.load_dataset` when that package is installed.
Text records need a tokenizer.  Sharding (`shard_index` / `num_shards`) strides records, the
way multiple producer replicas split one dataset.
"""

from __future__ import annotations

import json
from collections.abc import Iterable, Iterator
from pathlib import Path
from typing import Any

import numpy as np
import torch

TOKEN_KEYS = ("tokens", "input_ids")


def record_is_pretokenized(rec: Any) -> bool:
    """True when a dataset record already holds token ids (a tensor, an array, a list of ints or
    a dict with a "tokens" / "input_ids" field); False for text records."""
    if isinstance(rec, (torch.Tensor, np.ndarray)):
        return True
    if isinstance(rec, (list, tuple)):
        return not rec or isinstance(rec[0], (int, np.integer))
    if isinstance(rec, dict):
        return any(k in rec for k in TOKEN_KEYS)
    return False


def _record_tokens(rec: Any, tokenizer: Any, column: str = "text") -> torch.Tensor | None:
    if isinstance(rec, torch.Tensor):
        return rec.long().flatten()
    if isinstance(rec, np.ndarray):
        return torch.from_numpy(rec.astype(np.int64)).flatten()
    if isinstance(rec, (list, tuple)) and (not rec or isinstance(rec[0], (int, np.integer))):
        return torch.tensor(rec, dtype=torch.long)
    if isinstance(rec, str):
        rec = {column: rec}
    if isinstance(rec, dict):
        for k in TOKEN_KEYS:
            if k in rec:
                return torch.as_tensor(rec[k], dtype=torch.long).flatten()
        if column in rec:
            if tokenizer is None:
                raise ValueError("dataset has text records but no tokenizer was provided")
            return torch.tensor(tokenizer.encode(rec[column]), dtype=torch.long)
    raise ValueError(f"cannot interpret dataset record of type {type(rec)}")


def _iter_file(p: Path) -> Iterator[Any]:
    suf = p.suffix.lower()
    if suf == ".jsonl" or suf == ".json":
        with open(p) as f:
            for line in f:
                line = line.strip()
                if line:
                    yield json.loads(line)
    elif suf in (".parquet", ".arrow"):
        import pyarrow.parquet as pq

        if suf == ".parquet":
            table = pq.read_table(str(p))
        else:
            import pyarrow as pa

            with pa.memory_map(str(p)) as src:
                try:
                    table = pa.ipc.open_file(src).read_all()
                except pa.ArrowInvalid:
                    table = pa.ipc.open_stream(src).read_all()
        for batch in table.to_batches():
            for rec in batch.to_pylist():
                yield rec
    elif suf == ".npy":
        arr = np.load(p, mmap_mode="r")
        for row in arr:
            yield np.asarray(row)
    elif suf == ".pt":
        t = torch.load(p, map_location="cpu")
        for row in t:
            yield row
    else:
        raise ValueError(f"unsupported dataset file {p}")


def _iter_records(src: Any) -> Iterator[Any]:
    if isinstance(src, torch.Tensor):
        yield from (src if src.dim() > 1 else [src])
        return
    if isinstance(src, (str, Path)):
        s = str(src)
        p = Path(s)
        if p.is_dir():
            for f in sorted(p.iterdir()):
                if f.suffix.lower() in (".jsonl", ".json", ".parquet", ".arrow", ".npy", ".pt"):
                    yield from _iter_file(f)
            return
        if p.is_file():
            yield from _iter_file(p)
            return
        try:
            import datasets  # type: ignore[import-not-found]
        except ImportError as e:
            raise FileNotFoundError(f"dataset {s!r} is not a local path and HF datasets is not installed") from e
        yield from datasets.load_dataset(s, split="train", streaming=True)
        return
    yield from src


def synthetic_uniform(vocab: int, length: int, seed: int = 0) -> Iterator[torch.Tensor]:
    g = torch.Generator().manual_seed(seed)
    while True:
        yield torch.randint(0, vocab, (length,), generator=g)


def open_token_source(src: Any, tokenizer: Any = None, column: str = "text", shard_index: int = 0,
                      num_shards: int = 1, skip: int = 0, seed: int = 0, default_len: int = 1024,
                      with_kind: bool = False) -> Iterator[Any]:
    """Token sequences of `src`; with `with_kind`, (tokens, pretokenized) pairs, where
    `pretokenized` says whether the record already held token ids (synthetic sources do)."""
    if isinstance(src, str) and src.startswith("synthetic:"):
        parts = src.split(":")
        vocab = int(parts[2]) if len(parts) > 2 else 50257
        length = int(parts[3]) if len(parts) > 3 else default_len
        it: Iterable[torch.Tensor] = synthetic_uniform(vocab, length, seed=seed + 7919 * shard_index)
        for i, t in enumerate(it):
            if i >= skip:
                yield (t, True) if with_kind else t
        return
    for i, rec in enumerate(_iter_records(src)):
        if i % num_shards != shard_index:
            continue
        if i // num_shards < skip:
            continue
        t = _record_tokens(rec, tokenizer, column)
        if t is not None and t.numel() > 0:
            yield (t, record_is_pretokenized(rec)) if with_kind else t


def first_tokenized_length(src: Any) -> int | None:
    for rec in _iter_records(src):
        if isinstance(rec, dict):
            for k in TOKEN_KEYS:
                if k in rec:
                    return len(rec[k])
            return None
        try:
            return len(rec)
        except TypeError:
            return None
    return None
