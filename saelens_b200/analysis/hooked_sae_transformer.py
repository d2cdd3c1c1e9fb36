"""`HookedSAETransformer`: a producer LM into which SAEs are spliced at their hook points
(API of sae_lens/analysis/hooked_sae_transformer.py).

`add_sae(sae)` replaces the HookPoint named by `sae.cfg.metadata.hook_name` with a wrapper
that passes the activation through the SAE (encode -> decode).  With `use_error_term` the
wrapper adds back the SAE's reconstruction error, so downstream activations are unchanged while
the SAE's own hooks still see (and can edit) the features.  Transcoders read their input hook
and write their output hook.  `run_with_saes`, `run_with_cache_with_saes`,
`run_with_hooks_with_saes` attach SAEs for one call; `saes()` is the context-manager form and
puts back whatever SAEs were attached at those hooks before it (sae_lens/analysis/
hooked_sae_transformer.py:19-95 wrapper, 169-225 add / reset).  An unknown hook name or a reset
of a hook without an SAE logs a warning and changes nothing.

The error term is computed by a second, hook-free encode / decode of the same input, so an
intervention on the SAE's hooks (e.g. ablating `hook_sae_acts_post`) changes the reconstruction
but not the error.
"""

from __future__ import annotations

import logging
from collections.abc import Iterator
from contextlib import contextmanager
from typing import Any

import torch
from torch import nn

from saelens_b200.models.lm.transformer import HookedLM
from saelens_b200.models.sae import _disable_hooks
from saelens_b200.utils.hooks import HookPoint

logger = logging.getLogger(__name__)


class _SAEWrapper(nn.Module):
    """Sits where a HookPoint was: hook -> SAE -> output (optionally + error)."""

    def __init__(self, sae: Any, hook_point: HookPoint | None = None, use_error_term: bool = False):
        super().__init__()
        self.sae = sae
        self.hook_point = hook_point if hook_point is not None else HookPoint()
        self.use_error_term = use_error_term
        self.transcoder_input: torch.Tensor | None = None

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        x = self.hook_point(x)
        sae = self.sae
        src = (self.transcoder_input if self.transcoder_input is not None else x).to(sae.W_dec.dtype)
        dt = x.dtype
        y = sae.decode(sae.encode(src))
        if self.use_error_term:
            with torch.no_grad(), _disable_hooks(sae):
                clean = sae.decode(sae.encode(src))
            y = y + sae.hook_sae_error(x.to(clean.dtype) - clean)
        self.transcoder_input = None
        return sae.hook_sae_output(y).to(dt)


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
        """Splice `sae` at its hook (a transcoder: read its input hook, replace its output hook).
        `use_error_term` None takes the SAE's own setting."""
        err = bool(use_error_term if use_error_term is not None else getattr(sae, "use_error_term", False))
        self._attach(_SAEWrapper(sae, use_error_term=err))

    def _attach(self, wrapper: _SAEWrapper) -> None:
        sae = wrapper.sae
        hook = sae.cfg.metadata.hook_name
        out_hook = sae.cfg.metadata.hook_name_out or hook
        if out_hook not in self._acts_to_saes and out_hook not in self.hook_dict:
            logger.warning("No hook found for %s. Skipping. Check model.hook_dict for available hooks.", out_hook)
            return
        if out_hook in self._acts_to_saes:
            self._remove_one(out_hook)
        wrapper.hook_point = self.hook_dict[out_hook]
        _set_module(self, out_hook, wrapper)
        self._acts_to_saes[out_hook] = wrapper
        if out_hook != hook:  # transcoder: remember the input activation for the wrapper
            def grab(t: torch.Tensor, hook: HookPoint, w: _SAEWrapper = wrapper) -> None:
                w.transcoder_input = t
            in_hp = self.hook_dict[hook]
            in_hp.add_hook(grab, is_permanent=True)
            self._transcoder_in_handles[out_hook] = (in_hp, in_hp._fwd_handles[-1][0])
        self._rebuild_hook_dict()

    def _remove_one(self, out_hook: str) -> None:
        w = self._acts_to_saes.pop(out_hook)
        _set_module(self, out_hook, w.hook_point)
        grab = self._transcoder_in_handles.pop(out_hook, None)
        if grab is not None:  # only the input grab; other hooks on the input hook stay
            in_hp, handle = grab
            handle.remove()
            in_hp._fwd_handles = [e for e in in_hp._fwd_handles if e[0] is not handle]

    def _reset_sae(self, act_name: str, prev_wrapper: _SAEWrapper | None = None) -> None:
        """Remove the SAE at `act_name`; with `prev_wrapper`, attach that one in its place."""
        if act_name not in self._acts_to_saes:
            logger.warning("No SAE is attached to %s. There's nothing to reset.", act_name)
            return
        self._remove_one(act_name)
        if prev_wrapper is not None:
            self._attach(prev_wrapper)
        else:
            self._rebuild_hook_dict()

    def reset_saes(self, act_names: str | list[str] | None = None,
                   prev_wrappers: list[_SAEWrapper | None] | None = None) -> None:
        """Remove the SAEs at `act_names` (all by default); `prev_wrappers[i]`, when not None,
        is attached again in place of `act_names[i]`."""
        names = list(self._acts_to_saes) if act_names is None else ([act_names] if isinstance(act_names, str) else list(act_names))
        prev = prev_wrappers if prev_wrappers is not None else [None] * len(names)
        if len(prev) != len(names):
            raise ValueError("act_names and prev_wrappers must have the same length")
        for n, w in zip(names, prev):
            if n in self._acts_to_saes:
                self._reset_sae(n, w)
        self._rebuild_hook_dict()

    def _rebuild_hook_dict(self) -> None:
        self.setup()
        for name, w in self._acts_to_saes.items():
            self.hook_dict[name] = w.hook_point  # the LM's own hook keeps its name (and cache key)
            w.hook_point.name = name
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
        names: list[str] = []
        prev: list[_SAEWrapper | None] = []
        try:
            for s in saes:
                name = s.cfg.metadata.hook_name_out or s.cfg.metadata.hook_name
                names.append(name)
                prev.append(self._acts_to_saes.get(name))
                self.add_sae(s, use_error_term=use_error_term)
            yield self
        finally:
            if reset_saes_end:  # the SAEs attached before the context come back
                attached = [(n, p) for n, p in zip(names, prev) if n in self._acts_to_saes]
                self.reset_saes([n for n, _ in attached][::-1], [p for _, p in attached][::-1])

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
