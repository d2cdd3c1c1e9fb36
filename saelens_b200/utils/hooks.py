"""Named activation hooks (a self-contained replacement for TransformerLens hook points).

`HookPoint` is an identity module whose forward/backward hooks can be added by name;
`HookedRootModule` indexes every HookPoint below it by its dotted module path and offers
`run_with_hooks`, `run_with_cache` and a `hooks()` context manager.  The SAEs, the producer
language models and `HookedSAETransformer` all build on these two classes, mirroring the role
TransformerLens plays in the reference (sae_lens/saes/sae.py:26, load_model.py:130-309).
"""

from __future__ import annotations

from collections.abc import Callable, Iterable, Iterator, Sequence
from contextlib import contextmanager
from typing import Any

import torch
from torch import nn

HookFn = Callable[..., Any]
NameFilter = None | str | Sequence[str] | Callable[[str], bool]


class HookPoint(nn.Module):
    """Identity module with named forward (and backward) hooks."""

    def __init__(self) -> None:
        super().__init__()
        self.name: str | None = None
        self._fwd_handles: list[tuple[torch.utils.hooks.RemovableHandle, bool]] = []
        self._bwd_handles: list[tuple[torch.utils.hooks.RemovableHandle, bool]] = []

    def add_hook(self, hook: HookFn, dir: str = "fwd", is_permanent: bool = False,
                 prepend: bool = False) -> None:
        """`hook(tensor, hook=self)` may return a replacement tensor (forward only)."""
        if dir == "fwd":
            def _fwd(module: nn.Module, _inp: Any, out: torch.Tensor) -> Any:
                return hook(out, hook=module)

            handle = self.register_forward_hook(_fwd, prepend=prepend)
            self._fwd_handles.append((handle, is_permanent))
        elif dir == "bwd":
            def _bwd(module: nn.Module, grad_out: tuple[torch.Tensor, ...]) -> Any:
                res = hook(grad_out[0], hook=module)
                return None if res is None else (res,)

            handle = self.register_full_backward_pre_hook(_bwd, prepend=prepend)
            self._bwd_handles.append((handle, is_permanent))
        else:
            raise ValueError(f"dir must be 'fwd' or 'bwd', got {dir!r}")

    def remove_hooks(self, dir: str = "both", including_permanent: bool = False) -> None:
        def _strip(lst: list[tuple[torch.utils.hooks.RemovableHandle, bool]]):
            keep = []
            for h, perm in lst:
                if perm and not including_permanent:
                    keep.append((h, perm))
                else:
                    h.remove()
            return keep

        if dir in ("fwd", "both"):
            self._fwd_handles = _strip(self._fwd_handles)
        if dir in ("bwd", "both"):
            self._bwd_handles = _strip(self._bwd_handles)

    @property
    def has_hooks(self) -> bool:
        return bool(self._fwd_handles or self._bwd_handles)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return x


def _as_filter(names: NameFilter) -> Callable[[str], bool]:
    if names is None:
        return lambda _n: True
    if isinstance(names, str):
        return lambda n: n == names
    if callable(names):
        return names
    allowed = set(names)
    return lambda n: n in allowed


class HookedRootModule(nn.Module):
    """Base for modules whose HookPoints are addressed by dotted names."""

    def __init__(self) -> None:
        super().__init__()
        self.mod_dict: dict[str, nn.Module] = {}
        self.hook_dict: dict[str, HookPoint] = {}

    def setup(self) -> None:
        self.mod_dict = {}
        self.hook_dict = {}
        for name, mod in self.named_modules():
            if name == "":
                continue
            mod.name = name  # type: ignore[assignment]
            self.mod_dict[name] = mod
            if isinstance(mod, HookPoint):
                self.hook_dict[name] = mod

    def hook_points(self) -> Iterable[HookPoint]:
        return self.hook_dict.values()

    def add_hook(self, name: str | Callable[[str], bool], hook: HookFn, dir: str = "fwd",
                 is_permanent: bool = False, prepend: bool = False) -> None:
        if isinstance(name, str):
            if name not in self.hook_dict:
                raise KeyError(f"unknown hook point {name!r}")
            self.hook_dict[name].add_hook(hook, dir=dir, is_permanent=is_permanent, prepend=prepend)
            return
        for hp_name, hp in self.hook_dict.items():
            if name(hp_name):
                hp.add_hook(hook, dir=dir, is_permanent=is_permanent, prepend=prepend)

    def reset_hooks(self, including_permanent: bool = False, direction: str = "both") -> None:
        for hp in self.hook_dict.values():
            hp.remove_hooks(direction, including_permanent=including_permanent)

    @contextmanager
    def hooks(self, fwd_hooks: Sequence[tuple[Any, HookFn]] = (),
              bwd_hooks: Sequence[tuple[Any, HookFn]] = (),
              reset_hooks_end: bool = True) -> Iterator["HookedRootModule"]:
        try:
            for name, fn in fwd_hooks:
                self.add_hook(name, fn, dir="fwd")
            for name, fn in bwd_hooks:
                self.add_hook(name, fn, dir="bwd")
            yield self
        finally:
            if reset_hooks_end:
                self.reset_hooks(including_permanent=False)

    def run_with_hooks(self, *args: Any, fwd_hooks: Sequence[tuple[Any, HookFn]] = (),
                       bwd_hooks: Sequence[tuple[Any, HookFn]] = (),
                       reset_hooks_end: bool = True, **kwargs: Any) -> Any:
        with self.hooks(fwd_hooks, bwd_hooks, reset_hooks_end):
            return self(*args, **kwargs)

    def run_with_cache(self, *args: Any, names_filter: NameFilter = None,
                       remove_batch_dim: bool = False, **kwargs: Any) -> tuple[Any, dict[str, torch.Tensor]]:
        keep = _as_filter(names_filter)
        cache: dict[str, torch.Tensor] = {}

        def _save(t: torch.Tensor, hook: HookPoint) -> None:
            v = t.detach()
            cache[hook.name] = v[0] if remove_batch_dim else v  # type: ignore[index]

        fwd = [(n, _save) for n in self.hook_dict if keep(n)]
        with self.hooks(fwd_hooks=fwd):
            out = self(*args, **kwargs)
        return out, cache
