"""Cache LM activations to disk so SAE sweeps can skip the LM forward
(role of sae_lens/cache_activations_runner.py).

Writes `n_buffers` shards into `new_cached_activations_path`, each a safetensors file with
`activations` [n_seq, ctx, d_in] (the configured dtype) and `token_ids` [n_seq, ctx] (int32), plus
`cache_info.json` (hook, shapes, dtype, token counts).  Shards are written to a temporary
directory and moved into place at the end so a crashed run never leaves a half-written cache.
With `shuffle`, token rows are permuted across each shard before writing.
`ActivationsStore(..., cached_activations_path=...)` reads these shards back.
"""

from __future__ import annotations

import json
import shutil
from pathlib import Path
from typing import Any

import torch
from safetensors.torch import save_file

from saelens_b200.config import CacheActivationsRunnerConfig
from saelens_b200.training.activations_store import ActivationsStore
from saelens_b200.utils.misc import str_to_dtype


class CacheActivationsRunner:
    def __init__(self, cfg: CacheActivationsRunnerConfig, override_model: Any = None, override_dataset: Any = None):
        self.cfg = cfg
        if override_model is None:
            from saelens_b200.models.lm.load_model import load_model

            override_model = load_model(cfg.model_class_name, cfg.model_name, device=cfg.device,
                                        model_from_pretrained_kwargs=cfg.model_from_pretrained_kwargs)
        self.model = override_model
        self.store = ActivationsStore(
            model=self.model, dataset=override_dataset if override_dataset is not None else cfg.dataset_path,
            hook_name=cfg.hook_name, context_size=cfg.context_size, d_in=cfg.d_in,
            n_batches_in_buffer=cfg.n_batches_in_buffer, total_training_tokens=cfg.training_tokens,
            store_batch_size_prompts=cfg.model_batch_size, train_batch_size_tokens=cfg.n_tokens_in_batch,
            prepend_bos=cfg.prepend_bos, device=cfg.device, dtype=cfg.dtype, model_kwargs=cfg.model_kwargs,
            autocast_lm=cfg.autocast_lm, seqpos_slice=cfg.seqpos_slice, seed=cfg.seed,
        )

    def __str__(self) -> str:
        c = self.cfg
        return (f"CacheActivationsRunner(hook={c.hook_name}, d_in={c.d_in}, tokens={c.training_tokens}, "
                f"buffers={c.n_buffers} x {c.n_tokens_in_buffer} tokens, dtype={c.dtype})")

    @torch.no_grad()
    def _shard(self, n_seq: int) -> tuple[torch.Tensor, torch.Tensor]:
        acts, toks = [], []
        got = 0
        while got < n_seq:
            t = self.store.get_batch_tokens()
            a = self.store.get_activations(t)
            a = next(iter(a.values())) if isinstance(a, dict) else a
            if a.shape[-1] != self.cfg.d_in:
                raise RuntimeError(f"The hook {self.cfg.hook_name} has width {a.shape[-1]}, but d_in is "
                                   f"{self.cfg.d_in}: the cached activations would not match the config.")
            acts.append(a.to("cpu", str_to_dtype(self.cfg.dtype)))
            toks.append(t[:, slice(*self.cfg.seqpos_slice)].to(torch.int32).cpu())
            got += t.shape[0]
        A = torch.cat(acts)[:n_seq]
        T = torch.cat(toks)[:n_seq]
        if self.cfg.shuffle:
            g = torch.Generator().manual_seed(self.cfg.seed + n_seq)
            flatA = A.reshape(-1, A.shape[-1])
            flatT = T.reshape(-1)
            perm = torch.randperm(flatA.shape[0], generator=g)
            A = flatA[perm].reshape(A.shape)
            T = flatT[perm].reshape(T.shape)
        return A.contiguous(), T.contiguous()

    def run(self) -> Path:
        c = self.cfg
        out = Path(c.new_cached_activations_path or "activations")
        if out.exists() and any(out.iterdir()):  # never overwrite a directory the user filled
            raise FileExistsError(f"{out} is not empty. Please delete it or specify a different path.")
        tmp = out.parent / (out.name + ".tmp_shards")
        if tmp.exists():
            shutil.rmtree(tmp)
        tmp.mkdir(parents=True)
        seq_per_buffer = max(1, c.n_seq_in_buffer)
        remaining = c.n_seq_in_dataset
        i = 0
        total_tokens = 0
        while remaining > 0:
            n = min(seq_per_buffer, remaining)
            A, T = self._shard(n)
            save_file({"activations": A, "token_ids": T}, str(tmp / f"shard_{i:05d}.safetensors"))
            total_tokens += A.shape[0] * A.shape[1]
            remaining -= n
            i += 1
        info = {"hook_name": c.hook_name, "d_in": c.d_in, "context_size": c.sliced_context_size, "dtype": c.dtype,
                "n_shards": i, "total_tokens": total_tokens, "model_name": c.model_name, "dataset_path": c.dataset_path}
        (tmp / "cache_info.json").write_text(json.dumps(info, indent=2))
        if out.exists():  # an empty directory
            out.rmdir()
        tmp.rename(out)
        if c.hf_repo_id:
            self._push_to_hub(out)
        return out

    def _push_to_hub(self, path: Path) -> None:
        from huggingface_hub import HfApi

        api = HfApi()
        api.create_repo(self.cfg.hf_repo_id, repo_type="dataset", private=self.cfg.hf_is_private_repo, exist_ok=True)
        api.upload_folder(folder_path=str(path), repo_id=self.cfg.hf_repo_id, repo_type="dataset",
                          revision=self.cfg.hf_revision)
