"""`load_model`: resolve a producer LM by class name (interface of sae_lens/load_model.py:17-67).

* "HookedTransformer" / "HookedLM" / "HookedSAETransformer": this package's `HookedLM`; a preset
  name (e.g. "gpt2", "meta-llama/Meta-Llama-3-8B") gives a random-init model of that shape, a local
  Hugging Face checkpoint directory is converted weight for weight.
* "VLLMModel": the reference's vLLM activation producer (sae_lens/vllm_model.py:548).  Here it is
  this package's producer, `HookedLM`, resolved like "HookedTransformer": it runs to the hooked
  layer on the framework's own kernels (tcgen05 GEMMs and attention).  vLLM engine options
  (`gpu_memory_utilization`, `max_model_len`, `enforce_eager`, `tensor_parallel_size`, ...) have no
  meaning for it and are dropped; producer tensor parallelism is set by the runner's
  `vllm_tp_size`.
* "HookedMamba": needs the `mamba_lens` package, as in the reference.
* "AutoModelForCausalLM": a `transformers` model (local path, or `from_config` when
  `model_from_pretrained_kwargs={"random_init": True, ...config fields}`) wrapped in
  `HookedProxyLM`.
"""

from __future__ import annotations

from pathlib import Path
from typing import Any

import torch

from saelens_b200.models.lm.transformer import PRESETS, HookedLM


def _tokenizer(name: str) -> Any:
    try:
        from transformers import AutoTokenizer

        return AutoTokenizer.from_pretrained(name, local_files_only=True)
    except Exception:  # noqa: BLE001
        return None


# vLLM engine arguments a "VLLMModel" config may carry (sae_lens/vllm_model.py:548-625)
_VLLM_ENGINE_KWARGS = ("gpu_memory_utilization", "max_model_len", "enforce_eager", "tensor_parallel_size",
                       "pipeline_parallel_size", "distributed_executor_backend", "max_num_seqs",
                       "max_num_batched_tokens", "enable_chunked_prefill", "enable_prefix_caching", "seed_vllm",
                       "trust_remote_code", "swap_space", "kv_cache_dtype", "quantization", "n_devices")


def load_model(model_class_name: str, model_name: str, device: str | torch.device | None = None,
               model_from_pretrained_kwargs: dict[str, Any] | None = None) -> Any:
    kw = dict(model_from_pretrained_kwargs or {})
    if model_class_name == "VLLMModel":
        for k in _VLLM_ENGINE_KWARGS:
            kw.pop(k, None)
        model_class_name = "HookedTransformer"
    if model_class_name == "HookedMamba":
        try:
            from mamba_lens import HookedMamba  # type: ignore[import-not-found]
        except ImportError as e:
            raise ValueError("mamba-lens must be installed to load HookedMamba models") from e
        return HookedMamba.from_pretrained(model_name, device=device, **kw)
    kw.pop("n_devices", None)
    dtype = kw.pop("dtype", None)
    for ignored in ("center_writing_weights", "fold_ln", "center_unembed", "refactor_factored_attn_matrices"):
        kw.pop(ignored, None)
    if model_class_name in ("HookedTransformer", "HookedLM", "HookedSAETransformer"):
        cls: Any = HookedLM
        if model_class_name == "HookedSAETransformer":
            from saelens_b200.analysis.hooked_sae_transformer import HookedSAETransformer

            cls = HookedSAETransformer
        if Path(model_name).is_dir():
            from transformers import AutoModelForCausalLM

            from saelens_b200.models.lm.hf import hooked_lm_from_hf

            hf = AutoModelForCausalLM.from_pretrained(model_name, local_files_only=True)
            lm = hooked_lm_from_hf(hf, dtype=dtype, device=device)
            if cls is not HookedLM:
                lm.__class__ = cls
                cls._init_sae_state(lm)
            lm.tokenizer = _tokenizer(model_name)
            return lm
        if model_name not in PRESETS:
            raise ValueError(f"unknown model {model_name!r}: pass a preset ({sorted(PRESETS)}) or a local checkpoint dir")
        if dtype is not None:
            kw["dtype"] = dtype if isinstance(dtype, str) else str(dtype).replace("torch.", "")
        seed = kw.pop("seed", None)
        lm = cls.from_preset(model_name, device=device, seed=seed, **kw)
        lm.tokenizer = _tokenizer(model_name)
        return lm
    if model_class_name == "AutoModelForCausalLM":
        import transformers

        from saelens_b200.models.lm.hf import HookedProxyLM

        if kw.pop("random_init", False):
            cfg_cls = getattr(transformers, kw.pop("config_class", "LlamaConfig"))
            hf = transformers.AutoModelForCausalLM.from_config(cfg_cls(**kw))
        else:
            hf = transformers.AutoModelForCausalLM.from_pretrained(model_name, local_files_only=True, **kw)
        if dtype is not None:
            hf = hf.to(getattr(torch, dtype) if isinstance(dtype, str) else dtype)
        if device is not None:
            hf = hf.to(device)
        return HookedProxyLM(hf.eval(), tokenizer=_tokenizer(model_name))
    raise ValueError(f"Unknown model class: {model_class_name}")
