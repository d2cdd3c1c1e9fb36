"""Tokenize a text dataset once and store it as packed training contexts
(role of sae_lens/pretokenize_runner.py).

Records are tokenized, packed with the begin-batch / begin-sequence / separator rules of
`concat_and_batch_sequences`, optionally shuffled, and written as `tokens.npy` ([n, context_size]
int32) plus `sae_lens.json` metadata (tokenizer, context size, special-token settings) in
`save_path`; `hf_repo_id` uploads the folder with `huggingface_hub`.  The result is a valid
`dataset_path` for `LanguageModelSAERunnerConfig`.
"""

from __future__ import annotations

import json
from pathlib import Path
from typing import Any

import numpy as np
import torch

from saelens_b200 import __version__
from saelens_b200.config import PretokenizeRunnerConfig
from saelens_b200.training.datasets import open_token_source
from saelens_b200.training.tokenization_and_batching import concat_and_batch_sequences


def _special(tok: Any, tokenizer: Any) -> int | None:
    if tok is None or isinstance(tok, int):
        return tok
    return {"bos": tokenizer.bos_token_id, "eos": tokenizer.eos_token_id, "sep": tokenizer.sep_token_id}[tok]


def get_special_token_from_cfg(tok: Any, tokenizer: Any) -> int | None:
    return _special(tok, tokenizer)


class PretokenizeRunner:
    def __init__(self, cfg: PretokenizeRunnerConfig, tokenizer: Any = None, override_dataset: Any = None):
        self.cfg = cfg
        if tokenizer is None:
            from transformers import AutoTokenizer

            tokenizer = AutoTokenizer.from_pretrained(cfg.tokenizer_name, local_files_only=True)
        self.tokenizer = tokenizer
        self.dataset = override_dataset if override_dataset is not None else cfg.dataset_path

    def tokenize(self) -> np.ndarray:
        c = self.cfg
        if c.streaming and c.num_proc > 1:  # a streamed dataset is read by one process
            raise ValueError("num_proc must be 1 when streaming is True")
        src = open_token_source(self.dataset, tokenizer=self.tokenizer, column=c.column_name)
        rows = list(concat_and_batch_sequences(
            src, c.context_size, begin_batch_token_id=_special(c.begin_batch_token, self.tokenizer),
            begin_sequence_token_id=_special(c.begin_sequence_token, self.tokenizer),
            sequence_separator_token_id=_special(c.sequence_separator_token, self.tokenizer),
            disable_concat_sequences=c.disable_concat_sequences,
        ))
        arr = torch.stack(rows).to(torch.int32).numpy() if rows else np.zeros((0, c.context_size), np.int32)
        if c.shuffle and len(arr):
            rng = np.random.default_rng(c.seed)
            arr = arr[rng.permutation(len(arr))]
        return arr

    def metadata(self, n_rows: int) -> dict[str, Any]:
        c = self.cfg
        return {"sae_lens_version": __version__, "tokenizer_name": c.tokenizer_name, "original_dataset": c.dataset_path,
                "original_split": c.split, "original_data_files": c.data_files, "context_size": c.context_size,
                "shuffled": c.shuffle, "seed": c.seed, "begin_batch_token": c.begin_batch_token,
                "begin_sequence_token": c.begin_sequence_token, "sequence_separator_token": c.sequence_separator_token,
                "disable_concat_sequences": c.disable_concat_sequences, "n_rows": n_rows}

    def run(self) -> Path:
        arr = self.tokenize()
        if self.cfg.save_path is None and self.cfg.hf_repo_id is None:
            raise ValueError("set save_path or hf_repo_id")
        out = Path(self.cfg.save_path or f"pretokenized_{self.cfg.tokenizer_name.replace('/', '_')}")
        out.mkdir(parents=True, exist_ok=True)
        np.save(out / "tokens.npy", arr)
        (out / "sae_lens.json").write_text(json.dumps(self.metadata(len(arr)), indent=2))
        if self.cfg.hf_repo_id:
            from huggingface_hub import HfApi

            api = HfApi()
            api.create_repo(self.cfg.hf_repo_id, repo_type="dataset", private=self.cfg.hf_is_private_repo,
                            exist_ok=True)
            api.upload_folder(folder_path=str(out), repo_id=self.cfg.hf_repo_id, repo_type="dataset",
                              revision=self.cfg.hf_revision)
        return out


def pretokenize_runner(cfg: PretokenizeRunnerConfig) -> Path:
    return PretokenizeRunner(cfg).run()
