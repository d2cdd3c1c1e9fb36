"""`HookedSAETransformer`: a producer LM into which SAEs are spliced at their hook points
(API of sae_lens/analysis/hooked_sae_transformer.py).

`add_sae(sae)` replaces the HookPoint named by `sae.cfg.metadata.hook_name` with a wrapper
that passes the activation through the SAE (encode -> decode).  With `use_error_term` the
wrapper adds back the SAE's reconstruction error, so downstream activations are unchanged while
the SAE's own hooks still see (and can edit) the features.  Transcoders read their input hook
and write their output hook.  `run_with_saes`, `run_with_cache_with_saes`,
`run_with_hooks_with_saes` attach SAEs for one call; `saes()` is the context-manager form.
"""

from __future__ import annotations

from collections.abc import Iterator
from contextlib import contextmanager
from typing import Any

import torch
from torch import nn

from saelens_b200.models.lm.transformer import HookedLM
from saelens_b200.utils.hooks import HookPoint


class _SAEWrapper(nn.Module):
    """Sits where a HookPoint was: hook -> SAE -> output (optionally + error)."""

    def __init__(self, sae: Any, hook_point: HookPoint, use_error_term: bool = False):
        super().__init__()
        self.sae = sae
        self.hook_point = hook_point
        self.use_error_term = use_error_term
        self.transcoder_input: torch.Tensor | None = None

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        x = self.hook_point(x)
        src = self.transcoder_input if self.transcoder_input is not None else x
        dt = x.dtype
        y = self.sae(src.to(self.sae.W_dec.dtype))
        if self.use_error_term:
            with torch.no_grad():
                clean = self.sae.decode(self.sae.encode(src.to(self.sae.W_dec.dtype)))
            err = x.to(clean.dtype) - clean
            y = y + self.sae.hook_sae_error(err)
        self.transcoder_input = None
        return y.to(dt)


def _get_module(root: nn.Module, path: str) -> nn.Module:
    m = root
    for p in path.split("."):
        m = m[int(p)] if p.isdigit() else getattr(m, p)  # type: ignore[index]
    return m


def _set_module(root: nn.Module, path: str, new: nn.Module) -> None:
    parent_path, _, leaf = path.rpartition(".")
    parent = _get_module(root, parent_path) if parent_path else root
    if leaf.isdigit():
        parent[int(leaf)] = new  # type: ignore[index]
    else:
        setattr(parent, leaf, new)


class HookedSAETransformer(HookedLM):
    def __init__(self, *args: Any, **kwargs: Any):
        super().__init__(*args, **kwargs)
        self._init_sae_state(self)

    @staticmethod
    def _init_sae_state(obj: HookedLM) -> None:
        obj._acts_to_saes = {}  # type: ignore[attr-defined]
        obj._transcoder_in_handles = {}  # type: ignore[attr-defined]

    @property
    def acts_to_saes(self) -> dict[str, Any]:
        return {k: w.sae for k, w in self._acts_to_saes.items()}

    def add_sae(self, sae: Any, use_error_term: bool | None = None) -> None:
        hook = sae.cfg.metadata.hook_name
        out_hook = sae.cfg.metadata.hook_name_out or hook
        if out_hook not in self._acts_to_saes and out_hook not in self.hook_dict:
            raise ValueError(f"No hook found for {out_hook}")
        if out_hook in self._acts_to_saes:
            self._remove_one(out_hook)
        hp = self.hook_dict[out_hook]
        wrapper = _SAEWrapper(sae, hp, use_error_term=bool(use_error_term if use_error_term is not None
                                                           else getattr(sae, "use_error_term", False)))
        _set_module(self, out_hook, wrapper)
        self._acts_to_saes[out_hook] = wrapper
        if out_hook != hook:  # transcoder: remember the input activation for the wrapper
            def grab(t: torch.Tensor, hook: HookPoint, w: _SAEWrapper = wrapper) -> None:
                w.transcoder_input = t
            self.hook_dict[hook].add_hook(grab, is_permanent=True)
            self._transcoder_in_handles[out_hook] = hook
        self._rebuild_hook_dict()

    def _remove_one(self, out_hook: str) -> None:
        w = self._acts_to_saes.pop(out_hook)
        _set_module(self, out_hook, w.hook_point)
        in_hook = self._transcoder_in_handles.pop(out_hook, None)
        if in_hook is not None:
            self.hook_dict[in_hook].remove_hooks("fwd", including_permanent=True)

    def reset_saes(self, act_names: str | list[str] | None = None) -> None:
        names = list(self._acts_to_saes) if act_names is None else ([act_names] if isinstance(act_names, str) else act_names)
        for n in names:
            if n in self._acts_to_saes:
                self._remove_one(n)
        self._rebuild_hook_dict()

    def _rebuild_hook_dict(self) -> None:
        self.setup()
        for name, w in self._acts_to_saes.items():
            self.hook_dict[name] = w.hook_point
            for sname, hp in w.sae.hook_dict.items():
                self.hook_dict[f"{name}.{sname}"] = hp
                hp.name = f"{name}.{sname}"
        for name, mod in list(self.hook_dict.items()):
            if isinstance(mod, _SAEWrapper):
                self.hook_dict[name] = mod.hook_point

    def setup(self) -> None:
        super().setup()
        # SAE internals are re-registered under "<hook>.<sae hook>" by _rebuild_hook_dict
        for name in [n for n in self.hook_dict if ".sae." in n or n.endswith(".hook_point")]:
            del self.hook_dict[name]

    @contextmanager
    def saes(self, saes: Any = (), reset_saes_end: bool = True, use_error_term: bool | None = None) -> Iterator[HookedSAETransformer]:
        saes = [saes] if not isinstance(saes, (list, tuple)) else list(saes)
        try:
            for s in saes:
                self.add_sae(s, use_error_term=use_error_term)
            yield self
        finally:
            if reset_saes_end:
                self.reset_saes([s.cfg.metadata.hook_name_out or s.cfg.metadata.hook_name for s in saes])

    def run_with_saes(self, *args: Any, saes: Any = (), reset_saes_end: bool = True,
                      use_error_term: bool | None = None, **kwargs: Any) -> Any:
        with self.saes(saes, reset_saes_end=reset_saes_end, use_error_term=use_error_term):
            return self(*args, **kwargs)

    def run_with_cache_with_saes(self, *args: Any, saes: Any = (), reset_saes_end: bool = True,
                                 use_error_term: bool | None = None, **kwargs: Any) -> tuple[Any, dict[str, torch.Tensor]]:
        with self.saes(saes, reset_saes_end=reset_saes_end, use_error_term=use_error_term):
            return self.run_with_cache(*args, **kwargs)

    def run_with_hooks_with_saes(self, *args: Any, saes: Any = (), reset_saes_end: bool = True,
                                 fwd_hooks: Any = (), bwd_hooks: Any = (), reset_hooks_end: bool = True,
                                 **kwargs: Any) -> Any:
        with self.saes(saes, reset_saes_end=reset_saes_end):
            return self.run_with_hooks(*args, fwd_hooks=fwd_hooks, bwd_hooks=bwd_hooks,
                                       reset_hooks_end=reset_hooks_end, **kwargs)
