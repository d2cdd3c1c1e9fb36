"""Architecture name -> (SAE class, config class) maps for inference and training
(interface of sae_lens/registry.py:5-49)."""

from __future__ import annotations

from typing import Any

SAE_CLASS_REGISTRY: dict[str, tuple[type[Any], type[Any]]] = {}
SAE_TRAINING_CLASS_REGISTRY: dict[str, tuple[type[Any], type[Any]]] = {}


def register_sae_class(architecture: str, sae_class: type[Any], sae_config_class: type[Any]) -> None:
    if architecture in SAE_CLASS_REGISTRY:
        raise ValueError(f"SAE class for architecture {architecture} already registered.")
    SAE_CLASS_REGISTRY[architecture] = (sae_class, sae_config_class)


def register_sae_training_class(architecture: str, sae_training_class: type[Any],
                                sae_training_config_class: type[Any]) -> None:
    if architecture in SAE_TRAINING_CLASS_REGISTRY:
        raise ValueError(f"SAE training class for architecture {architecture} already registered.")
    SAE_TRAINING_CLASS_REGISTRY[architecture] = (sae_training_class, sae_training_config_class)


def get_sae_class(architecture: str) -> tuple[type[Any], type[Any]]:
    _ensure_builtin()
    try:
        return SAE_CLASS_REGISTRY[architecture]
    except KeyError as e:
        raise ValueError(
            f"unknown SAE architecture {architecture!r}; known: {sorted(SAE_CLASS_REGISTRY)}"
        ) from e


def get_sae_training_class(architecture: str) -> tuple[type[Any], type[Any]]:
    _ensure_builtin()
    try:
        return SAE_TRAINING_CLASS_REGISTRY[architecture]
    except KeyError as e:
        raise ValueError(
            f"unknown training SAE architecture {architecture!r}; known: "
            f"{sorted(SAE_TRAINING_CLASS_REGISTRY)}"
        ) from e


def _ensure_builtin() -> None:
    # importing the model package registers every built-in architecture exactly once
    import saelens_b200.models  # noqa: F401
