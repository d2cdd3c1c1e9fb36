"""`SAETransformerBridge`: the SAE-splicing API (`add_sae`, `run_with_saes`,
`run_with_cache_with_saes`, `run_with_hooks_with_saes`, `saes()`) for Hugging Face causal LMs
(role of sae_lens/analysis/sae_transformer_bridge.py, which targets TransformerLens v3's
`TransformerBridge`).

`boot_transformers` imports the Hugging Face model's weights into the framework's hooked
transformer (GPT-2 / Llama / Qwen2 / Gemma-2 families), whose modules carry the
TransformerLens hook names (`blocks.{i}.hook_resid_pre`, `...attn.hook_z`, ...), so SAEs
trained on those hook names splice in unchanged and the projections run on the tcgen05 GEMM.
"""

from __future__ import annotations

from typing import Any

from torch import nn

from saelens_b200.analysis.hooked_sae_transformer import HookedSAETransformer


def has_transformer_bridge() -> bool:
    """The bridge needs only `transformers` (no TransformerLens install); checked without importing it."""
    import importlib.util

    return importlib.util.find_spec("transformers") is not None


class SAETransformerBridge(HookedSAETransformer):
    @classmethod
    def boot_transformers(cls, model: str | nn.Module, *, device: Any = None, dtype: str | None = None,
                          tokenizer: Any = None, local_files_only: bool = True,
                          **from_pretrained_kwargs: Any) -> "SAETransformerBridge":
        from saelens_b200.models.lm.hf import hooked_lm_from_hf

        if isinstance(model, str):
            from transformers import AutoModelForCausalLM, AutoTokenizer

            name = model
            model = AutoModelForCausalLM.from_pretrained(name, local_files_only=local_files_only,
                                                         **from_pretrained_kwargs)
            if tokenizer is None:
                try:
                    tokenizer = AutoTokenizer.from_pretrained(name, local_files_only=local_files_only)
                except OSError:
                    tokenizer = None
        lm = hooked_lm_from_hf(model, dtype=dtype, device=device)
        lm.__class__ = cls
        cls._init_sae_state(lm)
        if tokenizer is not None:
            lm.tokenizer = tokenizer
        return lm  # type: ignore[return-value]
