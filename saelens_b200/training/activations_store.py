"""Produces training batches of LM activations at a hook point
(behaviour of sae_lens/training/activations_store.py, single-producer path).

tokens (packed contexts) -> LM forward that stops after the hooked layer -> activations at the
hook (optional head index, sequence-position slice, special-token filtering) -> mixing buffer ->
`train_batch_size_tokens` rows per `next()`.  Cached activations written by
`CacheActivationsRunner` can be read back instead of running the LM.  The dataset position is
saved in checkpoints so a resumed run continues where it stopped.
"""

from __future__ import annotations

import json
import warnings
from collections.abc import Iterator
from pathlib import Path
from typing import Any

import torch
from safetensors.torch import load_file, save_file

from saelens_b200.training.datasets import first_tokenized_length, open_token_source
from saelens_b200.training.mixing_buffer import mixing_buffer
from saelens_b200.training.tokenization_and_batching import concat_and_batch_sequences
from saelens_b200.utils.misc import extract_stop_at_layer_from_hook_name, get_special_token_ids, str_to_dtype


def _resolve_special(tok: Any, tokenizer: Any) -> int | None:
    if tok is None or isinstance(tok, int):
        return tok
    if tokenizer is None:
        return None
    return {"bos": getattr(tokenizer, "bos_token_id", None), "eos": getattr(tokenizer, "eos_token_id", None),
            "sep": getattr(tokenizer, "sep_token_id", None)}.get(tok)


class ActivationsStore:
    def __init__(self, model: Any, dataset: Any, hook_name: str, context_size: int, d_in: int,
                 n_batches_in_buffer: int, total_training_tokens: int, store_batch_size_prompts: int,
                 train_batch_size_tokens: int, prepend_bos: bool = True, normalize_activations: str = "none",
                 device: torch.device | str = "cpu", dtype: str | torch.dtype = "float32",
                 hook_head_index: int | None = None, cached_activations_path: str | None = None,
                 model_kwargs: dict[str, Any] | None = None, autocast_lm: bool = False,
                 seqpos_slice: tuple[int | None, ...] = (None,), exclude_special_tokens: bool | list[int] = False,
                 disable_concat_sequences: bool = False, sequence_separator_token: Any = "bos",
                 activations_mixing_fraction: float = 0.5, seed: int = 42, shard_index: int = 0, num_shards: int = 1,
                 hook_names: list[str] | None = None, tokenizer: Any = None, text_column: str = "text"):
        self.model = model
        self.hook_name = hook_name
        self.hook_names = hook_names or [hook_name]
        self.hook_head_index = hook_head_index
        self.context_size = context_size
        self.d_in = d_in
        self.n_batches_in_buffer = n_batches_in_buffer
        self.total_training_tokens = total_training_tokens
        self.store_batch_size_prompts = store_batch_size_prompts
        self.train_batch_size_tokens = train_batch_size_tokens
        self.prepend_bos = prepend_bos
        self.normalize_activations = normalize_activations
        self.device = torch.device(device)
        self.dtype = str_to_dtype(dtype) if isinstance(dtype, str) else dtype
        self.cached_activations_path = cached_activations_path
        self.model_kwargs = model_kwargs or {}
        self.autocast_lm = autocast_lm
        self.seqpos_slice = seqpos_slice
        self.disable_concat_sequences = disable_concat_sequences
        self.activations_mixing_fraction = activations_mixing_fraction
        self.shard_index, self.num_shards = shard_index, num_shards
        self.tokenizer = tokenizer if tokenizer is not None else getattr(model, "tokenizer", None)
        self.text_column = text_column
        self.dataset = dataset
        self.seed = seed
        self.n_dataset_processed = 0
        self.estimated_norm_scaling_factor: float | None = None
        if exclude_special_tokens is True:
            self.exclude_special_tokens: torch.Tensor | None = torch.tensor(
                get_special_token_ids(self.tokenizer) if self.tokenizer is not None else [], dtype=torch.long)
        elif isinstance(exclude_special_tokens, list):
            self.exclude_special_tokens = torch.tensor(exclude_special_tokens, dtype=torch.long)
        else:
            self.exclude_special_tokens = None
        bos = getattr(self.tokenizer, "bos_token_id", None) if self.tokenizer is not None else None
        self._begin_batch = bos if prepend_bos else None
        self._sep = _resolve_special(sequence_separator_token, self.tokenizer)
        self._stop_at = max(extract_stop_at_layer_from_hook_name(h) or 0 for h in self.hook_names) or None
        self._gen = torch.Generator().manual_seed(seed)
        self._cached_files: list[Path] = []
        if cached_activations_path is not None:
            self._cached_files = sorted(Path(cached_activations_path).glob("*.safetensors"))
            if not self._cached_files:
                raise FileNotFoundError(f"no activation shards in {cached_activations_path}")
        self._token_iter: Iterator[torch.Tensor] | None = None
        self._batch_iter: Iterator[Any] | None = None
        self._check_pretokenized_length()

    def _check_pretokenized_length(self) -> None:
        """A pretokenized dataset whose rows are shorter than `context_size` cannot fill a
        context (error); longer rows are cut to `context_size` (warning)."""
        if self.cached_activations_path is not None:
            return
        if isinstance(self.dataset, str) and self.dataset.startswith("synthetic:"):
            return
        if not isinstance(self.dataset, (str, Path, torch.Tensor, list, tuple)):  # one-shot iterables stay unread
            return
        try:
            n = first_tokenized_length(self.dataset)
        except (FileNotFoundError, ValueError, OSError):
            return
        if n is None:
            return
        if n < self.context_size:
            raise ValueError(f"pretokenized dataset has context size {n}, but the provided context_size is "
                             f"{self.context_size}: the dataset cannot fill a context.")
        if n > self.context_size:
            warnings.warn(f"pretokenized dataset has context size {n}, but the provided context_size is "
                          f"{self.context_size}; each row is cut to its first {self.context_size} tokens.", RuntimeWarning, stacklevel=3)

    # ---------------------------------------------------------------- construction helpers
    @classmethod
    def from_config(cls, model: Any, cfg: Any, override_dataset: Any = None, shard_index: int = 0,
                    num_shards: int = 1) -> ActivationsStore:
        ds = override_dataset if override_dataset is not None else cfg.dataset_path
        d_in = cfg.sae.d_in
        return cls(model=model, dataset=ds, hook_name=cfg.hook_name, hook_names=cfg.hook_names,
                   hook_head_index=cfg.hook_head_index, context_size=cfg.context_size, d_in=d_in,
                   n_batches_in_buffer=cfg.n_batches_in_buffer, total_training_tokens=cfg.training_tokens,
                   store_batch_size_prompts=cfg.store_batch_size_prompts,
                   train_batch_size_tokens=cfg.train_batch_size_tokens, prepend_bos=cfg.prepend_bos,
                   normalize_activations=cfg.sae.normalize_activations, device=cfg.act_store_device,
                   dtype=cfg.dtype, cached_activations_path=cfg.cached_activations_path if cfg.use_cached_activations else None,
                   model_kwargs=cfg.model_kwargs, autocast_lm=cfg.autocast_lm, seqpos_slice=cfg.seqpos_slice,
                   exclude_special_tokens=cfg.exclude_special_tokens,
                   disable_concat_sequences=cfg.disable_concat_sequences,
                   sequence_separator_token=cfg.sequence_separator_token,
                   activations_mixing_fraction=cfg.activations_mixing_fraction, seed=cfg.seed,
                   shard_index=shard_index, num_shards=num_shards)

    @classmethod
    def from_sae(cls, model: Any, sae: Any, dataset: Any, context_size: int | None = None,
                 store_batch_size_prompts: int = 8, train_batch_size_tokens: int = 4096, n_batches_in_buffer: int = 8,
                 total_tokens: int = 10**9, device: str = "cpu", dtype: str = "float32") -> ActivationsStore:
        md = sae.cfg.metadata
        return cls(model=model, dataset=dataset, hook_name=md.hook_name, hook_head_index=md.hook_head_index,
                   context_size=context_size or md.context_size or 128, d_in=sae.cfg.d_in,
                   n_batches_in_buffer=n_batches_in_buffer, total_training_tokens=total_tokens,
                   store_batch_size_prompts=store_batch_size_prompts, train_batch_size_tokens=train_batch_size_tokens,
                   prepend_bos=md.prepend_bos if md.prepend_bos is not None else True,
                   normalize_activations=sae.cfg.normalize_activations, device=device, dtype=dtype,
                   seqpos_slice=tuple(md.seqpos_slice) if md.seqpos_slice else (None,))

    # ---------------------------------------------------------------- tokens
    def _tokens(self) -> Iterator[torch.Tensor]:
        """Context-length token rows.  Pretokenized records are used as they are, each cut to
        `context_size` (their BOS / separator tokens were added when they were tokenized);
        text records are tokenized and packed with the BOS / separator rules
        (sae_lens/training/activations_store.py:499-530)."""
        src = open_token_source(self.dataset, tokenizer=self.tokenizer, column=self.text_column,
                                shard_index=self.shard_index, num_shards=self.num_shards,
                                skip=self.n_dataset_processed, seed=self.seed, default_len=self.context_size,
                                with_kind=True)
        try:
            first = next(src)
        except StopIteration:
            return iter(())

        def counted() -> Iterator[torch.Tensor]:
            self.n_dataset_processed += 1
            yield first[0]
            for t, _ in src:
                self.n_dataset_processed += 1
                yield t

        if first[1]:
            return (t[: self.context_size] for t in counted())
        return concat_and_batch_sequences(counted(), self.context_size, begin_batch_token_id=self._begin_batch,
                                          begin_sequence_token_id=None, sequence_separator_token_id=self._sep,
                                          disable_concat_sequences=self.disable_concat_sequences)

    def get_batch_tokens(self, batch_size: int | None = None) -> torch.Tensor:
        n = batch_size or self.store_batch_size_prompts
        if self._token_iter is None:
            self._token_iter = self._tokens()
        rows = []
        for _ in range(n):
            try:
                rows.append(next(self._token_iter))
            except StopIteration:
                self._token_iter = self._tokens()  # next epoch
                self.n_dataset_processed = 0
                rows.append(next(self._token_iter))
        return torch.stack(rows)

    # ---------------------------------------------------------------- activations
    @torch.no_grad()
    def get_activations(self, batch_tokens: torch.Tensor) -> torch.Tensor | dict[str, torch.Tensor]:
        """[B, S', d_in] activations for `batch_tokens` (dict by hook for several hooks)."""
        dev = getattr(self.model, "device", None) or next(self.model.parameters()).device
        ctx = torch.autocast(device_type=torch.device(dev).type, dtype=torch.bfloat16) if self.autocast_lm else _null()
        with ctx:
            _, cache = self.model.run_with_cache(batch_tokens.to(dev), names_filter=self.hook_names,
                                                 stop_at_layer=self._stop_at, **self.model_kwargs)
        out = {h: self._postprocess(cache[h]) for h in self.hook_names}
        return out if len(self.hook_names) > 1 else out[self.hook_name]

    def _postprocess(self, a: torch.Tensor) -> torch.Tensor:
        a = a[:, slice(*self.seqpos_slice)]
        if a.dim() == 4:  # [B, S, heads, d_head]
            a = a[:, :, self.hook_head_index] if self.hook_head_index is not None else a.flatten(-2)
        return a.to(device=self.device, dtype=self.dtype)

    def get_raw_llm_batch(self) -> tuple[torch.Tensor | dict[str, torch.Tensor], torch.Tensor]:
        toks = self.get_batch_tokens()
        acts = self.get_activations(toks)
        return acts, toks[:, slice(*self.seqpos_slice)]

    def get_filtered_llm_batch(self) -> torch.Tensor | dict[str, torch.Tensor]:
        acts, toks = self.get_raw_llm_batch()
        keep = None
        if self.exclude_special_tokens is not None and self.exclude_special_tokens.numel():
            keep = ~torch.isin(toks.reshape(-1), self.exclude_special_tokens)
        def flat(a: torch.Tensor) -> torch.Tensor:
            a = a.reshape(-1, a.shape[-1])
            return a[keep.to(a.device)] if keep is not None else a
        return {h: flat(v) for h, v in acts.items()} if isinstance(acts, dict) else flat(acts)

    @torch.no_grad()
    def get_streaming_activations(self, max_tokens: int) -> tuple[torch.Tensor, int]:
        """Up to `max_tokens` activation rows [n, d_in] for one streaming chunk (producer side of
        sae_lens/training/activations_store.py:778-915): whole LM batches are run, the rows past
        `max_tokens` are kept for the next chunk."""
        parts: list[torch.Tensor] = []
        have = 0
        rest = getattr(self, "_stream_residual", None)
        if rest is not None and rest.shape[0]:
            parts.append(rest)
            have = rest.shape[0]
        while have < max_tokens:
            a = self.get_filtered_llm_batch()
            if isinstance(a, dict):
                a = torch.cat([a[h] for h in self.hook_names], dim=-1)
            parts.append(a)
            have += a.shape[0]
        cat = torch.cat(parts) if len(parts) > 1 else parts[0]
        self._stream_residual = cat[max_tokens:]
        out = cat[:max_tokens]
        return out, int(out.shape[0])

    def _cached_batches(self) -> Iterator[torch.Tensor]:
        while True:
            for f in self._cached_files:
                sd = load_file(str(f))
                acts = sd["activations"]
                acts = acts.reshape(-1, acts.shape[-1]).to(device=self.device, dtype=self.dtype)
                for s in range(0, acts.shape[0], self.train_batch_size_tokens):
                    yield acts[s : s + self.train_batch_size_tokens]

    def _llm_batches(self) -> Iterator[Any]:
        if self._cached_files:
            yield from self._cached_batches()
            return
        while True:
            yield self.get_filtered_llm_batch()

    def _iterator(self) -> Iterator[Any]:
        buffer_tokens = self.n_batches_in_buffer * self.store_batch_size_prompts * self.context_size
        return mixing_buffer(buffer_size=max(buffer_tokens, self.train_batch_size_tokens),
                             batch_size=self.train_batch_size_tokens, activations_loader=self._llm_batches(),
                             mix_fraction=self.activations_mixing_fraction, generator=self._gen)

    def __iter__(self) -> ActivationsStore:
        return self

    def __next__(self) -> Any:
        if self._batch_iter is None:
            self._batch_iter = self._iterator()
        return next(self._batch_iter)

    def next_batch(self) -> Any:
        return next(self)

    # ---------------------------------------------------------------- checkpointing
    def state_dict(self) -> dict[str, torch.Tensor]:
        return {"n_dataset_processed": torch.tensor(self.n_dataset_processed)}

    def save_to_checkpoint(self, checkpoint_path: str | Path) -> None:
        from saelens_b200.constants import ACTIVATIONS_STORE_STATE_FILENAME

        save_file(self.state_dict(), str(Path(checkpoint_path) / ACTIVATIONS_STORE_STATE_FILENAME))

    def load_from_checkpoint(self, checkpoint_path: str | Path) -> None:
        from saelens_b200.constants import ACTIVATIONS_STORE_STATE_FILENAME

        sd = load_file(str(Path(checkpoint_path) / ACTIVATIONS_STORE_STATE_FILENAME))
        self.n_dataset_processed = int(sd["n_dataset_processed"].item())
        self._token_iter = None
        self._batch_iter = None

    def shuffle_input_dataset(self, seed: int) -> None:
        self.seed = seed
        self._token_iter = None
        self._batch_iter = None

    def reset_input_dataset(self) -> None:
        """Restart token reading from the first context (same seed), e.g. between eval passes.
        Activations already in the mixing buffer stay; later batches read the restarted tokens."""
        self.n_dataset_processed = 0
        self._token_iter = None

    def token_position(self) -> tuple[int, Any]:
        """Opaque token-reading position; `restore_token_position` puts it back."""
        return self.n_dataset_processed, self._token_iter

    def restore_token_position(self, pos: tuple[int, Any]) -> None:
        self.n_dataset_processed, self._token_iter = pos

    @torch.no_grad()
    def estimate_norm_scaling_factor(self, n_batches_for_norm_estimate: int = 100) -> float:
        norms = []
        for _ in range(n_batches_for_norm_estimate):
            a = self.get_filtered_llm_batch()
            a = next(iter(a.values())) if isinstance(a, dict) else a
            norms.append(a.float().norm(dim=-1).mean().item())
        self.estimated_norm_scaling_factor = (self.d_in ** 0.5) / (sum(norms) / len(norms))
        return self.estimated_norm_scaling_factor


class _null:
    def __enter__(self) -> None:
        return None

    def __exit__(self, *a: Any) -> None:
        return None


def write_dataset_metadata(path: Path, info: dict[str, Any]) -> None:
    (path / "sae_lens.json").write_text(json.dumps(info, indent=2))
