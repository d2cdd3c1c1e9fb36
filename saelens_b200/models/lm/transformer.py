"""Activation-producing language models with TransformerLens-style hook names.

One decoder-only implementation covers the producer families the reference drives (GPT-2
through TransformerLens; Llama / Mistral / Gemma-2 / Qwen2 through its vLLM fork, whose hook map
is sae_lens/vllm_model.py:235-364): learned or rotary positions, LayerNorm or RMSNorm, GELU or
gated (SwiGLU / GeGLU) MLPs, grouped-query attention with optional q/k/v bias, Gemma-2's
embedding scale, sandwich norms and logit soft-capping.

Hooks (per block i): `hook_resid_pre`, `ln1.hook_normalized`, `attn.hook_q/k/v` (before RoPE),
`attn.hook_z` (per-head attention output), `hook_attn_out`, `hook_resid_mid`, `ln2.hook_normalized`,
`mlp.hook_in` (the MLP's input), `mlp.hook_pre` (gate branch before the activation), `mlp.hook_post`, `hook_mlp_out`,
`hook_resid_post`; plus `hook_embed`, `hook_pos_embed`, `ln_final.hook_normalized`.
`run_with_cache(tokens, names_filter, stop_at_layer=n)` runs only blocks [0, n), which is how the
SAE data pipeline stops right after the hooked layer.

On CUDA with bf16 weights and no autograd, the forward runs on this package's kernels: the
q/k/v, output, MLP and unembedding projections on the tcgen05 GEMM (`saelens_b200.ops.gemm_tn`),
causal grouped-query attention (with Gemma-2's soft-cap) on the tcgen05 attention kernel
(`saelens_b200.ops.attention`), RMSNorm / LayerNorm, rotary embeddings, the gated activation and
the embedding gather on the elementwise kernels.  On CPU, or with autograd, the same math runs in
PyTorch (the CPU oracle of the tests).
"""

from __future__ import annotations

import contextlib

import math
from dataclasses import asdict, dataclass
from typing import Any

import torch
import torch.nn.functional as F
from torch import nn

from saelens_b200.utils.hooks import HookedRootModule, HookPoint


@dataclass
class LMConfig:
    n_layers: int
    d_model: int
    n_heads: int
    d_mlp: int
    d_vocab: int
    n_ctx: int
    d_head: int | None = None
    n_key_value_heads: int | None = None
    architecture: str = "llama"          # gpt2 | llama | gemma2 | qwen2 | mistral
    normalization: str = "RMS"            # LN | RMS
    positional: str = "rotary"            # standard | rotary
    act_fn: str = "silu"                  # gelu | gelu_new | gelu_pytorch_tanh | silu
    gated_mlp: bool = True
    qkv_bias: bool = False
    attn_out_bias: bool = False
    mlp_bias: bool = False
    rotary_base: float = 10000.0
    eps: float = 1e-5
    tie_embeddings: bool = False
    embed_scale: bool = False              # Gemma: embeddings * sqrt(d_model)
    sandwich_norm: bool = False            # Gemma-2: post-attention / post-MLP norms
    rms_one_plus: bool = False             # Gemma: weight applied as (1 + w)
    attn_softcap: float | None = None
    final_softcap: float | None = None
    query_pre_attn_scalar: float | None = None
    model_name: str = "custom"
    dtype: str = "bfloat16"
    init_std: float = 0.02

    def __post_init__(self) -> None:
        if self.d_head is None:
            self.d_head = self.d_model // self.n_heads
        if self.n_key_value_heads is None:
            self.n_key_value_heads = self.n_heads
        if self.n_heads % self.n_key_value_heads:
            raise ValueError("n_heads must be a multiple of n_key_value_heads")

    def to_dict(self) -> dict[str, Any]:
        return asdict(self)


def _preset(**kw: Any) -> LMConfig:
    return LMConfig(**kw)


PRESETS: dict[str, dict[str, Any]] = {
    # GPT-2 small
    "gpt2": dict(n_layers=12, d_model=768, n_heads=12, d_mlp=3072, d_vocab=50257, n_ctx=1024, architecture="gpt2",
                 normalization="LN", positional="standard", act_fn="gelu_new", gated_mlp=False, qkv_bias=True,
                 attn_out_bias=True, mlp_bias=True, tie_embeddings=True, model_name="gpt2"),
    "tiny-stories-1M": dict(n_layers=8, d_model=64, n_heads=16, d_mlp=256, d_vocab=50257, n_ctx=2048,
                            architecture="gpt2", normalization="LN", positional="standard", act_fn="gelu_new",
                            gated_mlp=False, qkv_bias=True, attn_out_bias=True, mlp_bias=True,
                            model_name="tiny-stories-1M"),
    "gelu-2l": dict(n_layers=2, d_model=512, n_heads=8, d_mlp=2048, d_vocab=48262, n_ctx=1024, architecture="gpt2",
                    normalization="LN", positional="standard", act_fn="gelu", gated_mlp=False, qkv_bias=True,
                    attn_out_bias=True, mlp_bias=True, model_name="gelu-2l"),
    # Llama-3-8B
    "meta-llama/Meta-Llama-3-8B": dict(n_layers=32, d_model=4096, n_heads=32, n_key_value_heads=8, d_mlp=14336,
                                       d_vocab=128256, n_ctx=8192, rotary_base=500000.0,
                                       model_name="meta-llama/Meta-Llama-3-8B"),
    "meta-llama/Llama-3.1-8B": dict(n_layers=32, d_model=4096, n_heads=32, n_key_value_heads=8, d_mlp=14336,
                                    d_vocab=128256, n_ctx=8192, rotary_base=500000.0,
                                    model_name="meta-llama/Llama-3.1-8B"),
    # Gemma-2-9B
    "google/gemma-2-9b": dict(n_layers=42, d_model=3584, n_heads=16, n_key_value_heads=8, d_head=256, d_mlp=14336,
                              d_vocab=256000, n_ctx=8192, architecture="gemma2", act_fn="gelu_pytorch_tanh",
                              embed_scale=True, sandwich_norm=True, rms_one_plus=True, eps=1e-6,
                              attn_softcap=50.0, final_softcap=30.0, query_pre_attn_scalar=256.0,
                              tie_embeddings=True, model_name="google/gemma-2-9b"),
    # Qwen-14B (Qwen1.5 / Qwen2 layout)
    "Qwen/Qwen1.5-14B": dict(n_layers=40, d_model=5120, n_heads=40, d_mlp=13696, d_vocab=152064, n_ctx=8192,
                             architecture="qwen2", qkv_bias=True, rotary_base=1000000.0, eps=1e-6,
                             model_name="Qwen/Qwen1.5-14B"),
    "Qwen/Qwen2.5-14B": dict(n_layers=48, d_model=5120, n_heads=40, n_key_value_heads=8, d_mlp=13824,
                             d_vocab=152064, n_ctx=8192, architecture="qwen2", qkv_bias=True,
                             rotary_base=1000000.0, eps=1e-6, model_name="Qwen/Qwen2.5-14B"),
}
PRESETS["gpt2-small"] = PRESETS["gpt2"]
PRESETS["llama-3-8b"] = PRESETS["meta-llama/Meta-Llama-3-8B"]
PRESETS["gemma-2-9b"] = PRESETS["google/gemma-2-9b"]
PRESETS["qwen-14b"] = PRESETS["Qwen/Qwen2.5-14B"]


def preset_config(name: str, **overrides: Any) -> LMConfig:
    if name not in PRESETS:
        raise KeyError(f"unknown model preset {name!r}; known: {sorted(PRESETS)}")
    return LMConfig(**{**PRESETS[name], **overrides})


# ------------------------------------------------------------------------------ layers
class NativeLinear(nn.Module):
    """y = x W^T + b with W [out, in]; the tcgen05 GEMM on CUDA bf16 (any width; the input width a
    multiple of 8 elements, i.e. 16-byte rows)."""

    def __init__(self, d_in: int, d_out: int, bias: bool, dtype: torch.dtype, device: Any = None):
        super().__init__()
        self.weight = nn.Parameter(torch.empty(d_out, d_in, dtype=dtype, device=device))
        self.bias = nn.Parameter(torch.zeros(d_out, dtype=dtype, device=device)) if bias else None
        self._native_ok = d_in % 8 == 0
        self._bias_f32: torch.Tensor | None = None

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        w = self.weight
        if (self._native_ok and x.is_cuda and w.dtype == torch.bfloat16 and x.dtype == torch.bfloat16
                and not torch.is_grad_enabled() and not FORCE_TORCH):
            from saelens_b200 import ops

            if ops.available():
                shp = x.shape
                x2 = x.reshape(-1, shp[-1])
                if not x2.is_contiguous():
                    x2 = x2.contiguous()
                b = None
                if self.bias is not None:
                    if self._bias_f32 is None or self._bias_f32.device != w.device:
                        self._bias_f32 = self.bias.detach().float().contiguous()
                    b = self._bias_f32
                out, _ = ops.gemm_tn(x2, w, bias=b, status=_status_for(x2))
                if not out.is_contiguous():  # a width that is not a multiple of 8
                    out = out.contiguous()
                return out.view(*shp[:-1], w.shape[0])
        return F.linear(x, w, self.bias)

    def _load_from_state_dict(self, *args: Any, **kwargs: Any) -> None:
        self._bias_f32 = None
        super()._load_from_state_dict(*args, **kwargs)


class _FusedWeights:
    """Row-concatenation of several projections' weights (and fp32 biases), rebuilt whenever one of
    them changes (storage or in-place version), so one tcgen05 GEMM computes all of them."""

    def __init__(self) -> None:
        self._key: tuple | None = None
        self.w: torch.Tensor | None = None
        self.b: torch.Tensor | None = None

    def get(self, layers: list[NativeLinear]) -> tuple[torch.Tensor, torch.Tensor | None]:
        params = [p for m in layers for p in ((m.weight,) if m.bias is None else (m.weight, m.bias))]
        key = tuple((p.data_ptr(), p._version) for p in params)
        if key != self._key:
            self.w = torch.cat([m.weight.detach() for m in layers]).contiguous()
            has_b = any(m.bias is not None for m in layers)
            self.b = torch.cat([m.bias.detach().float() if m.bias is not None else
                                torch.zeros(m.weight.shape[0], device=m.weight.device) for m in layers]) if has_b else None
            self._key = key
        assert self.w is not None
        return self.w, self.b


def _fused_linear(x: torch.Tensor, cache: _FusedWeights, layers: list[NativeLinear]) -> torch.Tensor:
    """[..., sum of the layers' widths] output of one tcgen05 GEMM over the concatenated weights."""
    from saelens_b200 import ops

    w, b = cache.get(layers)
    x2 = x.reshape(-1, x.shape[-1])
    if not x2.is_contiguous():
        x2 = x2.contiguous()
    out, _ = ops.gemm_tn(x2, w, bias=b, status=_status_for(x2))
    return out.view(*x.shape[:-1], w.shape[0]) if out.is_contiguous() else out.reshape(*x.shape[:-1], w.shape[0])


def _tied_unembed(x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    """x @ w.T with the embedding matrix (tied unembedding) on the tcgen05 GEMM when possible."""
    if x.dtype == torch.bfloat16 and w.dtype == torch.bfloat16 and x.shape[-1] % 8 == 0 and _native_ok(x):
        from saelens_b200 import ops

        x2 = x.reshape(-1, x.shape[-1]).contiguous()
        out, _ = ops.gemm_tn(x2, w, status=_status_for(x2))
        return out.contiguous().view(*x.shape[:-1], w.shape[0])
    return x @ w.T


# Set to True to run the producer on PyTorch ops even on CUDA (the comparison arm of the
# producer timing case); never needed otherwise.
FORCE_TORCH = False

# One device status word per CUDA device for the producer's kernels: the GEMMs and attention
# report a timed-out wait there, and HookedLM.forward reads it once per forward instead of each
# kernel reading its own (a device synchronisation per call, which would drain the launch queue
# between every projection).
_STATUS: dict[torch.device, Any] = {}


def _status_for(t: torch.Tensor):
    st = _STATUS.get(t.device)
    if st is None:
        from saelens_b200.ops import StatusWord

        st = _STATUS[t.device] = StatusWord(t.device)
    return st


def _native_ok(t: torch.Tensor) -> bool:
    """Use the framework's CUDA kernels for inference-mode producer ops on a CUDA tensor."""
    if FORCE_TORCH or not (t.is_cuda and not torch.is_grad_enabled()):
        return False
    from saelens_b200 import ops

    return ops.available()


class Norm(nn.Module):
    def __init__(self, cfg: LMConfig, dtype: torch.dtype):
        super().__init__()
        self.rms = cfg.normalization == "RMS"
        self.eps = cfg.eps
        self.one_plus = cfg.rms_one_plus
        self.w = nn.Parameter(torch.zeros(cfg.d_model, dtype=dtype) if self.one_plus else torch.ones(cfg.d_model, dtype=dtype))
        self.b = None if self.rms else nn.Parameter(torch.zeros(cfg.d_model, dtype=dtype))
        self.hook_normalized = HookPoint()

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if (self.rms and x.dtype in (torch.bfloat16, torch.float32) and x.dtype == self.w.dtype
                and x.shape[-1] % 8 == 0 and _native_ok(x)):
            from saelens_b200.ops import native

            x2 = x.reshape(-1, x.shape[-1])
            if not x2.is_contiguous():
                x2 = x2.contiguous()
            y = native().rmsnorm(x2, self.w, self.eps, self.one_plus).view(x.shape)
            return self.hook_normalized(y)
        if (not self.rms and x.dtype in (torch.bfloat16, torch.float32) and x.dtype == self.w.dtype
                and x.shape[-1] % 8 == 0 and _native_ok(x)):
            from saelens_b200.ops import native

            x2 = x.reshape(-1, x.shape[-1])
            if not x2.is_contiguous():
                x2 = x2.contiguous()
            y = native().layernorm(x2, self.w, self.b, self.eps).view(x.shape)
            return self.hook_normalized(y)
        xf = x.float()
        if self.rms:
            y = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + self.eps)
            w = (1.0 + self.w.float()) if self.one_plus else self.w.float()
            y = y * w
        else:
            y = F.layer_norm(xf, (xf.shape[-1],), self.w.float(), self.b.float() if self.b is not None else None, self.eps)
        return self.hook_normalized(y.to(x.dtype))


def _act(name: str, x: torch.Tensor) -> torch.Tensor:
    if name == "silu":
        return F.silu(x)
    if name in ("gelu_new", "gelu_pytorch_tanh"):
        return F.gelu(x, approximate="tanh")
    if name == "gelu":
        return F.gelu(x)
    if name == "relu":
        return F.relu(x)
    raise ValueError(f"unknown activation {name}")


def rotary_tables(n_pos: int, d: int, base: float, device: Any, dtype: torch.dtype = torch.float32):
    inv = 1.0 / (base ** (torch.arange(0, d, 2, device=device, dtype=torch.float32) / d))
    t = torch.arange(n_pos, device=device, dtype=torch.float32)
    f = torch.outer(t, inv)
    return torch.cos(f).to(dtype), torch.sin(f).to(dtype)


def apply_rotary(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """x [B, S, H, d]; rotate-half convention (first half paired with second half)."""
    if x.dtype == torch.bfloat16 and cos.dtype == torch.float32 and _native_ok(x):
        from saelens_b200.ops import native

        y = x.contiguous().clone() if x.is_contiguous() else x.contiguous()
        native().rope_(y, cos.contiguous(), sin.contiguous(), 0)
        return y
    d2 = x.shape[-1] // 2
    x1, x2 = x[..., :d2].float(), x[..., d2:].float()
    c = cos[None, :, None, :]
    s = sin[None, :, None, :]
    return torch.cat([x1 * c - x2 * s, x2 * c + x1 * s], dim=-1).to(x.dtype)


class Attention(nn.Module):
    def __init__(self, cfg: LMConfig, dtype: torch.dtype):
        super().__init__()
        self.cfg = cfg
        H, KV, dh = cfg.n_heads, cfg.n_key_value_heads, cfg.d_head
        assert dh is not None and KV is not None
        self.q = NativeLinear(cfg.d_model, H * dh, cfg.qkv_bias, dtype)
        self.k = NativeLinear(cfg.d_model, KV * dh, cfg.qkv_bias, dtype)
        self.v = NativeLinear(cfg.d_model, KV * dh, cfg.qkv_bias, dtype)
        self.o = NativeLinear(H * dh, cfg.d_model, cfg.attn_out_bias, dtype)
        self.hook_q, self.hook_k, self.hook_v = HookPoint(), HookPoint(), HookPoint()
        self.hook_z = HookPoint()
        self.hook_rot_q, self.hook_rot_k = HookPoint(), HookPoint()
        self.scale = 1.0 / math.sqrt(cfg.query_pre_attn_scalar if cfg.query_pre_attn_scalar else dh)
        self._qkv = _FusedWeights()
        # tensor parallelism (models/lm/tp.py): this rank's heads and the group
        self.n_heads_local, self.n_kv_local = H, KV
        self.tp: Any = None
        self.o_bias_after: torch.Tensor | None = None

    def _hook(self, hp: HookPoint, t: torch.Tensor, dim: int) -> torch.Tensor:
        """Run a hook point on a head-sharded tensor: under tensor parallelism, a hook that is
        attached sees the full width (all-gathered along `dim`) and the rank keeps its shard of
        the result."""
        if self.tp is None or not hp.has_hooks:
            return hp(t)
        return self.tp.hooked(hp, t, dim)

    def forward(self, x: torch.Tensor, rot: tuple[torch.Tensor, torch.Tensor] | None) -> torch.Tensor:
        B, S, _ = x.shape
        H, KV, dh = self.n_heads_local, self.n_kv_local, self.cfg.d_head
        fused = (x.dtype == torch.bfloat16 and self.q.weight.dtype == torch.bfloat16 and x.shape[-1] % 8 == 0
                 and _native_ok(x))
        if fused:
            # one GEMM for q, k and v; the heads are strided views of its output
            qkv = _fused_linear(x, self._qkv, [self.q, self.k, self.v])
            q = self._hook(self.hook_q, qkv[..., : H * dh].view(B, S, H, dh), 2)
            k = self._hook(self.hook_k, qkv[..., H * dh : (H + KV) * dh].view(B, S, KV, dh), 2)
            v = self._hook(self.hook_v, qkv[..., (H + KV) * dh :].view(B, S, KV, dh), 2)
        else:
            q = self._hook(self.hook_q, self.q(x).view(B, S, H, dh), 2)
            k = self._hook(self.hook_k, self.k(x).view(B, S, KV, dh), 2)
            v = self._hook(self.hook_v, self.v(x).view(B, S, KV, dh), 2)
        if rot is not None:
            in_place = (fused and rot[0].dtype == torch.float32 and not (self.hook_q.has_hooks or self.hook_k.has_hooks)
                        and q.stride(-1) == 1 and k.stride(-1) == 1)
            if in_place:
                # nothing holds the pre-rotation values: rotate q and k where they are
                from saelens_b200.ops import native

                cos, sin = rot[0].contiguous(), rot[1].contiguous()
                native().rope_(q, cos, sin, 0)
                native().rope_(k, cos, sin, 0)
                q, k = self._hook(self.hook_rot_q, q, 2), self._hook(self.hook_rot_k, k, 2)
            else:
                q = self._hook(self.hook_rot_q, apply_rotary(q, *rot), 2)
                k = self._hook(self.hook_rot_k, apply_rotary(k, *rot), 2)
        if q.dtype == torch.bfloat16 and dh in (64, 128, 256) and _native_ok(q):
            from saelens_b200 import ops

            # tcgen05 prefill attention: K/V heads are read in place by their query-head group,
            # the soft-cap (Gemma-2) is applied to the logits inside the kernel
            z = ops.attention(q, k, v, self.scale, softcap=self.cfg.attn_softcap, causal=True,
                              status=_status_for(q))
            z = self._hook(self.hook_z, z, 2)
            return self._out(z.reshape(B, S, H * dh))
        qh, kh, vh = q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2)
        if KV != H:
            rep = H // KV
            kh = kh.repeat_interleave(rep, dim=1)
            vh = vh.repeat_interleave(rep, dim=1)
        if self.cfg.attn_softcap:
            sc = (qh.float() @ kh.float().transpose(-1, -2)) * self.scale
            sc = self.cfg.attn_softcap * torch.tanh(sc / self.cfg.attn_softcap)
            mask = torch.ones(S, S, dtype=torch.bool, device=x.device).tril()
            sc = sc.masked_fill(~mask, float("-inf"))
            z = (torch.softmax(sc, dim=-1) @ vh.float()).to(x.dtype)
        else:
            z = F.scaled_dot_product_attention(qh, kh, vh, is_causal=True, scale=self.scale)
        z = self._hook(self.hook_z, z.transpose(1, 2), 2)  # [B, S, H, dh]
        return self._out(z.reshape(B, S, H * dh))

    def _out(self, z: torch.Tensor) -> torch.Tensor:
        """Output projection; under tensor parallelism the partial sums of the ranks' heads are
        all-reduced and the bias is added once, after the sum."""
        y = self.o(z)
        if self.tp is not None:
            y = self.tp.all_reduce(y)
            if self.o_bias_after is not None:
                y = y + self.o_bias_after
        return y


class MLP(nn.Module):
    def __init__(self, cfg: LMConfig, dtype: torch.dtype):
        super().__init__()
        self.cfg = cfg
        self.gated = cfg.gated_mlp
        if self.gated:
            self.gate = NativeLinear(cfg.d_model, cfg.d_mlp, cfg.mlp_bias, dtype)
        self.up = NativeLinear(cfg.d_model, cfg.d_mlp, cfg.mlp_bias, dtype)
        self.down = NativeLinear(cfg.d_mlp, cfg.d_model, cfg.mlp_bias, dtype)
        self.hook_in = HookPoint()  # the MLP's input (after the pre-MLP norm): transcoders read it
        self.hook_pre = HookPoint()
        self.hook_post = HookPoint()
        self._gate_up = _FusedWeights()
        self.d_mlp_local = cfg.d_mlp
        self.tp: Any = None
        self.down_bias_after: torch.Tensor | None = None

    def _hook(self, hp: HookPoint, t: torch.Tensor) -> torch.Tensor:
        if self.tp is None or not hp.has_hooks:
            return hp(t)
        return self.tp.hooked(hp, t, t.dim() - 1)

    def _down(self, post: torch.Tensor) -> torch.Tensor:
        y = self.down(post)
        if self.tp is not None:
            y = self.tp.all_reduce(y)
            if self.down_bias_after is not None:
                y = y + self.down_bias_after
        return y

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        x = self.hook_in(x)
        if self.gated:
            kind = {"silu": 0, "gelu_new": 1, "gelu_pytorch_tanh": 1}.get(self.cfg.act_fn)
            d = self.d_mlp_local
            if (kind is not None and x.dtype == torch.bfloat16 and self.gate.weight.dtype == torch.bfloat16
                    and x.shape[-1] % 8 == 0 and d % 8 == 0 and _native_ok(x)):
                # one GEMM for the gate and up projections; the activation reads both halves in place
                from saelens_b200.ops import native

                gu = _fused_linear(x, self._gate_up, [self.gate, self.up])
                pre = self._hook(self.hook_pre, gu[..., :d])
                up = gu[..., d:]
                if pre.shape == up.shape and pre.stride(-1) == 1:
                    post = self._hook(self.hook_post, native().gated_act(pre, up, kind))
                else:
                    post = self._hook(self.hook_post, _act(self.cfg.act_fn, pre) * up)
                return self._down(post)
            pre = self._hook(self.hook_pre, self.gate(x))
            up = self.up(x)
            if kind is not None and pre.dtype == torch.bfloat16 and pre.shape == up.shape and _native_ok(pre):
                from saelens_b200.ops import native

                post = self._hook(self.hook_post, native().gated_act(pre.contiguous(), up.contiguous(), kind))
            else:
                post = self._hook(self.hook_post, _act(self.cfg.act_fn, pre) * up)
        else:
            pre = self._hook(self.hook_pre, self.up(x))
            post = self._hook(self.hook_post, _act(self.cfg.act_fn, pre))
        return self._down(post)


class Block(nn.Module):
    def __init__(self, cfg: LMConfig, dtype: torch.dtype):
        super().__init__()
        self.cfg = cfg
        self.ln1 = Norm(cfg, dtype)
        self.attn = Attention(cfg, dtype)
        self.ln2 = Norm(cfg, dtype)
        self.mlp = MLP(cfg, dtype)
        if cfg.sandwich_norm:
            self.ln1_post = Norm(cfg, dtype)
            self.ln2_post = Norm(cfg, dtype)
        self.hook_resid_pre = HookPoint()
        self.hook_attn_out = HookPoint()
        self.hook_resid_mid = HookPoint()
        self.hook_mlp_out = HookPoint()
        self.hook_resid_post = HookPoint()

    def forward(self, x: torch.Tensor, rot: tuple[torch.Tensor, torch.Tensor] | None) -> torch.Tensor:
        x = self.hook_resid_pre(x)
        a = self.attn(self.ln1(x), rot)
        if self.cfg.sandwich_norm:
            a = self.ln1_post(a)
        a = self.hook_attn_out(a)
        x = self.hook_resid_mid(x + a)
        m = self.mlp(self.ln2(x))
        if self.cfg.sandwich_norm:
            m = self.ln2_post(m)
        m = self.hook_mlp_out(m)
        return self.hook_resid_post(x + m)


class HookedLM(HookedRootModule):
    """Decoder-only LM whose activations can be cached or edited by hook name."""

    def __init__(self, cfg: LMConfig, device: Any = None, init: bool = True, tokenizer: Any = None):
        super().__init__()
        self.cfg = cfg
        dtype = getattr(torch, cfg.dtype)
        # parameters are allocated and initialised on `device` directly (an 8B-parameter model
        # built on the host first would spend minutes in host RNG and copies)
        with torch.device(device) if device is not None else contextlib.nullcontext():
            self.embed = nn.Embedding(cfg.d_vocab, cfg.d_model, dtype=dtype)
            self.hook_embed = HookPoint()
            if cfg.positional == "standard":
                self.pos_embed = nn.Embedding(cfg.n_ctx, cfg.d_model, dtype=dtype)
                self.hook_pos_embed = HookPoint()
            self.blocks = nn.ModuleList([Block(cfg, dtype) for _ in range(cfg.n_layers)])
            self.ln_final = Norm(cfg, dtype)
            self.unembed = None if cfg.tie_embeddings else NativeLinear(cfg.d_model, cfg.d_vocab, False, dtype)
            self.tokenizer = tokenizer
            self._rot: tuple[torch.Tensor, torch.Tensor] | None = None
            if init:
                self.init_weights()
        if device is not None:
            self.to(device)
        self.setup()

    # ---------------------------------------------------------------- construction
    @classmethod
    def from_preset(cls, name: str, device: Any = None, seed: int | None = None, **overrides: Any) -> HookedLM:
        if seed is not None:
            torch.manual_seed(seed)
        return cls(preset_config(name, **overrides), device=device)

    @torch.no_grad()
    def init_weights(self) -> None:
        std = self.cfg.init_std
        for name, p in self.named_parameters():
            if p.dim() >= 2:
                p.normal_(0.0, std)
                if name.endswith(("o.weight", "down.weight")):
                    p.mul_(1.0 / math.sqrt(2 * self.cfg.n_layers))
            elif name.endswith(".b") or name.endswith("bias"):
                p.zero_()

    @property
    def W_U(self) -> torch.Tensor:
        return self.embed.weight if self.unembed is None else self.unembed.weight

    @property
    def device(self) -> torch.device:
        return self.embed.weight.device

    # ---------------------------------------------------------------- forward
    def _rotary(self, S: int) -> tuple[torch.Tensor, torch.Tensor] | None:
        if self.cfg.positional != "rotary":
            return None
        dev = self.embed.weight.device
        if self._rot is None or self._rot[0].shape[0] < S or self._rot[0].device != dev:
            self._rot = rotary_tables(max(S, self.cfg.n_ctx), self.cfg.d_head or 0, self.cfg.rotary_base, dev)
        return self._rot[0][:S], self._rot[1][:S]

    def _embed(self, tokens: torch.Tensor) -> torch.Tensor:
        """Token embedding (times sqrt(d_model) for Gemma) plus learned positions when present.
        With no hooks on `hook_embed` / `hook_pos_embed` the gather, scale and position add are one
        kernel on CUDA."""
        S = tokens.shape[1]
        w = self.embed.weight
        hooked = self.hook_embed.has_hooks or (self.cfg.positional == "standard" and self.hook_pos_embed.has_hooks)
        if (not hooked and w.dtype in (torch.bfloat16, torch.float32) and w.shape[1] % 8 == 0 and _native_ok(w)):
            from saelens_b200.ops import native

            scale = math.sqrt(self.cfg.d_model) if self.cfg.embed_scale else 1.0
            if scale != 1.0 and w.dtype == torch.bfloat16:
                scale = float(torch.tensor(scale, dtype=torch.bfloat16))  # the eager path's bf16 constant
            pos = self.pos_embed.weight if self.cfg.positional == "standard" else None
            bad = torch.zeros(1, dtype=torch.int32, device=w.device)
            x = native().embed(tokens.contiguous(), w, scale, pos, bad)
            self._bad_tokens = bad
            return x
        x = self.hook_embed(self.embed(tokens))
        if self.cfg.embed_scale:
            x = x * torch.tensor(math.sqrt(self.cfg.d_model), dtype=x.dtype, device=x.device)
        if self.cfg.positional == "standard":
            pos = torch.arange(S, device=tokens.device)
            x = x + self.hook_pos_embed(self.pos_embed(pos))[None]
        return x

    def forward(self, tokens: torch.Tensor, return_type: str | None = "logits",
                stop_at_layer: int | None = None, start_at_layer: int | None = None,
                residual: torch.Tensor | None = None) -> torch.Tensor | None:
        out = self._forward(tokens, return_type, stop_at_layer, start_at_layer, residual)
        dev = self.embed.weight.device
        if dev in _STATUS:
            _STATUS[dev].check("producer LM forward")
        return out

    def _forward(self, tokens: torch.Tensor, return_type: str | None, stop_at_layer: int | None,
                 start_at_layer: int | None, residual: torch.Tensor | None) -> torch.Tensor | None:
        if isinstance(tokens, str) or (isinstance(tokens, list) and tokens and isinstance(tokens[0], str)):
            tokens = self.to_tokens(tokens)
        if start_at_layer is None:
            tokens = tokens.to(self.embed.weight.device)
            if tokens.dim() == 1:
                tokens = tokens.unsqueeze(0)
            S = tokens.shape[1]
            x = self._embed(tokens)
            start = 0
        else:
            assert residual is not None
            x, S, start = residual, residual.shape[1], start_at_layer
        rot = self._rotary(S)
        end = self.cfg.n_layers if stop_at_layer is None else min(stop_at_layer, self.cfg.n_layers)
        for blk in self.blocks[start:end]:
            x = blk(x, rot)
        if stop_at_layer is not None and stop_at_layer < self.cfg.n_layers:
            return x
        if return_type is None:
            return None
        x = self.ln_final(x)
        if return_type == "residual":
            return x
        logits = _tied_unembed(x, self.W_U) if self.unembed is None else self.unembed(x)
        if self.cfg.final_softcap:
            logits = self.cfg.final_softcap * torch.tanh(logits.float() / self.cfg.final_softcap)
        if return_type == "logits":
            return logits
        if return_type == "loss":
            return self.loss_fn(logits, tokens)
        if return_type == "both":
            return logits, self.loss_fn(logits, tokens)  # type: ignore[return-value]
        raise ValueError(f"unknown return_type {return_type}")

    @staticmethod
    def loss_fn(logits: torch.Tensor, tokens: torch.Tensor, per_token: bool = False) -> torch.Tensor:
        lp = torch.log_softmax(logits.float(), dim=-1)[:, :-1]
        nll = -lp.gather(-1, tokens[:, 1:].unsqueeze(-1)).squeeze(-1)
        return nll if per_token else nll.mean()

    # ---------------------------------------------------------------- tokenizer helpers
    def to_tokens(self, text: str | list[str], prepend_bos: bool = True, truncate: bool = True) -> torch.Tensor:
        if self.tokenizer is None:
            raise ValueError("this model has no tokenizer attached")
        texts = [text] if isinstance(text, str) else text
        ids = [self.tokenizer.encode(t) for t in texts]
        bos = getattr(self.tokenizer, "bos_token_id", None)
        if prepend_bos and bos is not None:
            ids = [[bos] + i for i in ids]
        if truncate:
            ids = [i[: self.cfg.n_ctx] for i in ids]
        L = max(len(i) for i in ids)
        pad = getattr(self.tokenizer, "pad_token_id", None) or 0
        out = torch.full((len(ids), L), pad, dtype=torch.long)
        for r, i in enumerate(ids):
            out[r, : len(i)] = torch.tensor(i)
        return out.to(self.device)

    def to_string(self, tokens: torch.Tensor) -> str | list[str]:
        if self.tokenizer is None:
            raise ValueError("this model has no tokenizer attached")
        if tokens.dim() == 1:
            return self.tokenizer.decode(tokens.tolist())
        return [self.tokenizer.decode(t.tolist()) for t in tokens]
