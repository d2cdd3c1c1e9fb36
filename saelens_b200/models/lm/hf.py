"""Hugging Face `transformers` models as activation producers.

* `HookedProxyLM` wraps any causal LM: every submodule's output gets a HookPoint named by its
  module path, `run_with_cache(..., stop_at_layer=n)` raises a private exception right after
  decoder layer n-1 so the rest of the network never runs (role of sae_lens/load_model.py:130-309).
* `hooked_lm_from_hf` converts Llama / Mistral / Qwen2 / Gemma-2 / GPT-2 checkpoints into this
  package's `HookedLM`, whose projections run on the native GEMM.
"""

from __future__ import annotations

import re
from typing import Any

import torch
from torch import nn

from saelens_b200.models.lm.transformer import HookedLM, LMConfig
from saelens_b200.utils.hooks import HookedRootModule, HookPoint, NameFilter, _as_filter


class _StopForward(Exception):
    pass


class HookedProxyLM(HookedRootModule):
    """TransformerLens-like hooks over an arbitrary HF causal LM."""

    def __init__(self, model: nn.Module, tokenizer: Any = None):
        super().__init__()
        self.model = model
        self.tokenizer = tokenizer
        self._proxy_hooks: dict[str, HookPoint] = {}
        self._layer_names: list[str] = []
        for name, mod in model.named_modules():
            if name == "":
                continue
            hp = HookPoint()
            hp.name = name
            self._proxy_hooks[name] = hp
            mod.register_forward_hook(self._make_fwd(name))
            if re.fullmatch(r".*layers\.\d+|.*\.h\.\d+", name):
                self._layer_names.append(name)
        self.hook_dict = dict(self._proxy_hooks)
        self._stop_after: str | None = None

    def setup(self) -> None:  # hooks are managed explicitly
        pass

    def _make_fwd(self, name: str):
        def fwd(_mod: nn.Module, _inp: Any, out: Any) -> Any:
            hp = self._proxy_hooks[name]
            if hp.has_hooks:
                t = out[0] if isinstance(out, tuple) else out
                if isinstance(t, torch.Tensor):
                    new = hp(t)
                    if isinstance(out, tuple):
                        out = (new, *out[1:])
                    else:
                        out = new
            if self._stop_after == name:
                raise _StopForward
            return out

        return fwd

    @property
    def cfg(self) -> Any:
        return self.model.config

    def forward(self, tokens: torch.Tensor, return_type: str | None = "logits", stop_at_layer: int | None = None,
                **kwargs: Any) -> Any:
        """`return_type` "logits" (or None) gives the logits; "both" gives (logits, loss) with the
        Hugging Face model's own next-token loss and cannot stop early (sae_lens/load_model.py
        HookedProxyLM.forward)."""
        if return_type not in ("logits", "both", None):
            raise NotImplementedError(f"Only return_type supported is 'both', 'logits' or None, got {return_type!r}")
        if return_type == "both" and stop_at_layer is not None:
            raise NotImplementedError("stop_at_layer is not supported for return_type='both'")
        kwargs.pop("_names_filter", None)
        if stop_at_layer is not None and 0 < stop_at_layer <= len(self._layer_names):
            self._stop_after = self._layer_names[stop_at_layer - 1]
        dev = next(self.model.parameters()).device
        try:
            if return_type == "both":
                ids = tokens.to(dev)
                out = self.model(input_ids=ids, labels=ids, **kwargs)
                return _extract_logits_from_output(out), out.loss
            return _extract_logits_from_output(self.model(input_ids=tokens.to(dev), **kwargs))
        except _StopForward:
            return None
        finally:
            self._stop_after = None

    def run_with_cache(self, *args: Any, names_filter: NameFilter = None, remove_batch_dim: bool = False,
                       **kwargs: Any) -> tuple[Any, dict[str, torch.Tensor]]:
        keep = _as_filter(names_filter)
        cache: dict[str, torch.Tensor] = {}

        def save(t: torch.Tensor, hook: HookPoint) -> None:
            cache[hook.name] = (t[0] if remove_batch_dim else t).detach()  # type: ignore[index]

        fwd = [(n, save) for n in self._proxy_hooks if keep(n)]
        with self.hooks(fwd_hooks=fwd):
            out = self(*args, **kwargs)
        return out, cache

    def to_tokens(self, text: str | list[str], prepend_bos: bool | None = False, padding_side: str | None = None,
                  truncate: bool = False, move_to_device: bool = False) -> torch.Tensor:
        """Tokenizer ids exactly as the Hugging Face tokenizer makes them: the tokenizer decides
        about BOS, so the TransformerLens-style options are accepted only at their no-op values."""
        if prepend_bos is not False:
            raise ValueError("Only works with prepend_bos=False, to match the Hugging Face tokenizer")
        if padding_side is not None:
            raise ValueError("Only works with padding_side=None, to match the Hugging Face tokenizer")
        if truncate:
            raise ValueError("Only works with truncate=False, to match the Hugging Face tokenizer")
        if move_to_device:
            raise ValueError("Only works with move_to_device=False, to match the Hugging Face tokenizer")
        enc = self.tokenizer(text if isinstance(text, list) else [text], return_tensors="pt", padding=True)
        return enc["input_ids"]


def _extract_logits_from_output(out: Any) -> torch.Tensor | None:
    """Logits from a Hugging Face model output: a tensor, a dict-like or object with `logits`
    (None when it is None), or a tuple whose first entry is the logits."""
    if isinstance(out, torch.Tensor):
        return out
    if isinstance(out, dict):
        return out.get("logits")
    if isinstance(out, tuple):
        return out[0]
    if hasattr(out, "logits"):
        return out.logits
    raise ValueError(f"Unsupported model output type: {type(out)}")


def _cfg_from_hf(hc: Any) -> LMConfig:
    mt = getattr(hc, "model_type", "llama")
    if mt == "gpt2":
        return LMConfig(n_layers=hc.n_layer, d_model=hc.n_embd, n_heads=hc.n_head, d_mlp=hc.n_inner or 4 * hc.n_embd,
                        d_vocab=hc.vocab_size, n_ctx=hc.n_positions, architecture="gpt2", normalization="LN",
                        positional="standard", act_fn="gelu_new", gated_mlp=False, qkv_bias=True,
                        attn_out_bias=True, mlp_bias=True, eps=hc.layer_norm_epsilon, tie_embeddings=True,
                        model_name=getattr(hc, "_name_or_path", "gpt2") or "gpt2", dtype="float32")
    kw: dict[str, Any] = dict(
        n_layers=hc.num_hidden_layers, d_model=hc.hidden_size, n_heads=hc.num_attention_heads,
        n_key_value_heads=getattr(hc, "num_key_value_heads", None) or hc.num_attention_heads,
        d_head=getattr(hc, "head_dim", None) or hc.hidden_size // hc.num_attention_heads,
        d_mlp=hc.intermediate_size, d_vocab=hc.vocab_size, n_ctx=getattr(hc, "max_position_embeddings", 2048),
        rotary_base=float(getattr(hc, "rope_theta", None) or (getattr(hc, "rope_parameters", None) or {}).get("rope_theta", 10000.0)),
        eps=getattr(hc, "rms_norm_eps", 1e-6), tie_embeddings=bool(getattr(hc, "tie_word_embeddings", False)),
        model_name=getattr(hc, "_name_or_path", mt) or mt, dtype="float32",
    )
    if mt in ("qwen2",):
        kw.update(architecture="qwen2", qkv_bias=True)
    elif mt in ("gemma2",):
        kw.update(architecture="gemma2", act_fn="gelu_pytorch_tanh", embed_scale=True, sandwich_norm=True,
                  rms_one_plus=True, attn_softcap=getattr(hc, "attn_logit_softcapping", None),
                  final_softcap=getattr(hc, "final_logit_softcapping", None),
                  query_pre_attn_scalar=getattr(hc, "query_pre_attn_scalar", None))
    else:
        kw.update(architecture=mt if mt in ("llama", "mistral") else "llama",
                  qkv_bias=bool(getattr(hc, "attention_bias", False)))
    return LMConfig(**kw)


@torch.no_grad()
def hooked_lm_from_hf(hf_model: nn.Module, dtype: str | None = None, device: Any = None) -> HookedLM:
    hc = hf_model.config
    cfg = _cfg_from_hf(hc)
    if dtype is not None:
        cfg.dtype = dtype
    lm = HookedLM(cfg, init=False)
    sd = hf_model.state_dict()
    t = lambda k: sd[k]  # noqa: E731
    if cfg.architecture == "gpt2":
        p = "transformer."
        lm.embed.weight.copy_(t(p + "wte.weight"))
        lm.pos_embed.weight.copy_(t(p + "wpe.weight"))
        for i, b in enumerate(lm.blocks):
            q = f"{p}h.{i}."
            b.ln1.w.copy_(t(q + "ln_1.weight")); b.ln1.b.copy_(t(q + "ln_1.bias"))
            b.ln2.w.copy_(t(q + "ln_2.weight")); b.ln2.b.copy_(t(q + "ln_2.bias"))
            W = t(q + "attn.c_attn.weight")  # Conv1D: [d_model, 3 d_model]
            bb = t(q + "attn.c_attn.bias")
            d = cfg.d_model
            for j, lin in enumerate((b.attn.q, b.attn.k, b.attn.v)):
                lin.weight.copy_(W[:, j * d : (j + 1) * d].T)
                lin.bias.copy_(bb[j * d : (j + 1) * d])
            b.attn.o.weight.copy_(t(q + "attn.c_proj.weight").T); b.attn.o.bias.copy_(t(q + "attn.c_proj.bias"))
            b.mlp.up.weight.copy_(t(q + "mlp.c_fc.weight").T); b.mlp.up.bias.copy_(t(q + "mlp.c_fc.bias"))
            b.mlp.down.weight.copy_(t(q + "mlp.c_proj.weight").T); b.mlp.down.bias.copy_(t(q + "mlp.c_proj.bias"))
        lm.ln_final.w.copy_(t(p + "ln_f.weight")); lm.ln_final.b.copy_(t(p + "ln_f.bias"))
    else:
        p = "model."
        lm.embed.weight.copy_(t(p + "embed_tokens.weight"))
        for i, b in enumerate(lm.blocks):
            q = f"{p}layers.{i}."
            b.ln1.w.copy_(t(q + "input_layernorm.weight"))
            b.attn.q.weight.copy_(t(q + "self_attn.q_proj.weight"))
            b.attn.k.weight.copy_(t(q + "self_attn.k_proj.weight"))
            b.attn.v.weight.copy_(t(q + "self_attn.v_proj.weight"))
            b.attn.o.weight.copy_(t(q + "self_attn.o_proj.weight"))
            if cfg.qkv_bias:
                b.attn.q.bias.copy_(t(q + "self_attn.q_proj.bias"))
                b.attn.k.bias.copy_(t(q + "self_attn.k_proj.bias"))
                b.attn.v.bias.copy_(t(q + "self_attn.v_proj.bias"))
            b.mlp.gate.weight.copy_(t(q + "mlp.gate_proj.weight"))
            b.mlp.up.weight.copy_(t(q + "mlp.up_proj.weight"))
            b.mlp.down.weight.copy_(t(q + "mlp.down_proj.weight"))
            if cfg.sandwich_norm:
                b.ln1_post.w.copy_(t(q + "post_attention_layernorm.weight"))
                b.ln2.w.copy_(t(q + "pre_feedforward_layernorm.weight"))
                b.ln2_post.w.copy_(t(q + "post_feedforward_layernorm.weight"))
            else:
                b.ln2.w.copy_(t(q + "post_attention_layernorm.weight"))
        lm.ln_final.w.copy_(t(p + "norm.weight"))
        if lm.unembed is not None:
            lm.unembed.weight.copy_(t("lm_head.weight"))
    if dtype is not None:
        lm.to(getattr(torch, dtype))
    if device is not None:
        lm.to(device)
    lm.setup()
    return lm
