"""Loaders that turn on-disk or Hugging Face SAE checkpoints into (cfg_dict, state_dict).

Covers the native layout (`cfg.json` + `sae_weights.safetensors`) and third-party layouts that
need a weight-name / shape conversion (interface of sae_lens/loading/pretrained_sae_loaders.py:
loaders take `(repo_id, folder_name, device, force_download, cfg_overrides)` and return
`(cfg_dict, state_dict, log_sparsity | None)`; disk loaders take `(path, device, cfg_overrides)`).
Configs written before the 6.0 layout are migrated by `handle_config_defaulting`.
"""

from __future__ import annotations

import json
import re
from collections.abc import Callable
from pathlib import Path
from typing import Any

import numpy as np
import torch
from packaging.version import InvalidVersion, Version
from safetensors import safe_open

from saelens_b200.constants import (
    SAE_CFG_FILENAME,
    SAE_WEIGHTS_FILENAME,
    SPARSIFY_WEIGHTS_FILENAME,
    SPARSITY_FILENAME,
)
from saelens_b200.registry import get_sae_class
from saelens_b200.utils.misc import filter_valid_dataclass_fields, str_to_dtype

# Loader signatures (the interface third-party converters implement)
PretrainedSaeHuggingfaceLoader = Callable[..., "tuple[dict[str, Any], dict[str, torch.Tensor], torch.Tensor | None]"]
PretrainedSaeDiskLoader = Callable[..., "tuple[dict[str, Any], dict[str, torch.Tensor]]"]
PretrainedSaeConfigHuggingfaceLoader = Callable[..., dict[str, Any]]

LLM_METADATA_KEYS = {
    "model_name", "hook_name", "model_class_name", "hook_head_index", "model_from_pretrained_kwargs",
    "prepend_bos", "exclude_special_tokens", "neuronpedia_id", "context_size", "seqpos_slice",
    "dataset_path", "sae_lens_version", "sae_lens_training_version", "hook_name_out",
    "hook_head_index_out", "hf_hook_name", "hf_hook_name_out",
}


try:  # a file missing from a hub repo, or from the local cache when offline
    from huggingface_hub.errors import EntryNotFoundError as _EntryNotFound

    MISSING_FILE_ERRORS: tuple[type[BaseException], ...] = (OSError, _EntryNotFound)
except ImportError:
    MISSING_FILE_ERRORS = (OSError,)


def _hf_download(repo_id: str, filename: str, force_download: bool = False, subfolder: str | None = None) -> str:
    from huggingface_hub import hf_hub_download

    return hf_hub_download(repo_id=repo_id, filename=filename, subfolder=subfolder,
                           force_download=force_download)


def load_safetensors_weights(path: str | Path, device: str = "cpu",
                             dtype: torch.dtype | str | None = None) -> dict[str, torch.Tensor]:
    dt = str_to_dtype(dtype) if dtype is not None else None
    out: dict[str, torch.Tensor] = {}
    with safe_open(str(path), framework="pt", device=device) as f:  # type: ignore[no-untyped-call]
        for k in f.keys():  # noqa: SIM118
            t = f.get_tensor(k)
            out[k] = t.to(dtype=dt) if dt is not None else t
    return out


def read_sae_components_from_disk(cfg_dict: dict[str, Any], weight_path: str | Path, device: str = "cpu",
                                  dtype: torch.dtype | None = None) -> tuple[dict[str, Any], dict[str, torch.Tensor]]:
    dt = dtype or str_to_dtype(cfg_dict.get("dtype", "float32"))
    sd = load_safetensors_weights(weight_path, device=device, dtype=dt)
    _handle_scaling_factor(cfg_dict, sd)
    return cfg_dict, sd


def _handle_scaling_factor(cfg_dict: dict[str, Any], sd: dict[str, torch.Tensor]) -> None:
    if "scaling_factor" not in sd:
        cfg_dict["finetuning_scaling_factor"] = False
        return
    sf = sd.pop("scaling_factor")
    if torch.allclose(sf, torch.ones_like(sf)):
        cfg_dict["finetuning_scaling_factor"] = False
        return
    if not cfg_dict.get("finetuning_scaling_factor"):
        raise ValueError("Scaling factor is present but finetuning_scaling_factor is False.")
    sd["finetuning_scaling_factor"] = sf


# ------------------------------------------------------------------------------ native layout
def get_sae_lens_config_from_disk(path: str | Path, device: str | None = None,
                                  cfg_overrides: dict[str, Any] | None = None) -> dict[str, Any]:
    with open(Path(path) / SAE_CFG_FILENAME) as f:
        cfg = json.load(f)
    if device is not None:
        cfg["device"] = device
    if cfg_overrides:
        cfg.update(cfg_overrides)
    return cfg


def sae_lens_disk_loader(path: str | Path, device: str = "cpu",
                         cfg_overrides: dict[str, Any] | None = None) -> tuple[dict[str, Any], dict[str, torch.Tensor]]:
    cfg = get_sae_lens_config_from_disk(path, device, cfg_overrides)
    return read_sae_components_from_disk(cfg, Path(path) / SAE_WEIGHTS_FILENAME, device=device)


def get_sae_lens_config_from_hf(repo_id: str, folder_name: str, device: str | None = None,
                                force_download: bool = False,
                                cfg_overrides: dict[str, Any] | None = None) -> dict[str, Any]:
    p = _hf_download(repo_id, f"{folder_name}/{SAE_CFG_FILENAME}", force_download)
    return get_sae_lens_config_from_disk(Path(p).parent, device, cfg_overrides)


def sae_lens_huggingface_loader(repo_id: str, folder_name: str, device: str = "cpu", force_download: bool = False,
                                cfg_overrides: dict[str, Any] | None = None):
    cfg = get_sae_lens_config_from_hf(repo_id, folder_name, device, force_download, cfg_overrides)
    wpath = _hf_download(repo_id, f"{folder_name}/{SAE_WEIGHTS_FILENAME}", force_download)
    try:
        spath: str | None = _hf_download(repo_id, f"{folder_name}/{SPARSITY_FILENAME}", force_download)
    except MISSING_FILE_ERRORS:
        spath = None
    cfg, sd = read_sae_components_from_disk(cfg, wpath, device=device)
    log_sparsity = None
    if spath is not None:
        with safe_open(spath, framework="pt", device=device) as f:  # type: ignore[no-untyped-call]
            log_sparsity = f.get_tensor("sparsity")
    return cfg, sd, log_sparsity


# ------------------------------------------------------------------------------ config migration
def handle_config_defaulting(cfg_dict: dict[str, Any]) -> dict[str, Any]:
    version = cfg_dict.get("sae_lens_version")
    if not version and isinstance(cfg_dict.get("metadata"), dict):
        version = cfg_dict["metadata"].get("sae_lens_version")
    try:
        old = (not version) or Version(str(version)) < Version("6.0.0-rc.0")
    except InvalidVersion:
        old = False
    if old and "metadata" not in cfg_dict:
        return handle_pre_6_0_config(cfg_dict)
    return cfg_dict


def handle_pre_6_0_config(cfg_dict: dict[str, Any]) -> dict[str, Any]:
    """Rename pre-6.0 keys, fill their defaults and move LM fields into `metadata`."""
    renames = {"hook_point": "hook_name", "hook_point_head_index": "hook_head_index",
               "activation_fn_str": "activation_fn"}
    cfg = {renames.get(k, k): v for k, v in cfg_dict.items()}
    cfg.setdefault("prepend_bos", True)
    cfg.setdefault("dataset_trust_remote_code", True)
    cfg.setdefault("apply_b_dec_to_input", True)
    cfg.setdefault("finetuning_scaling_factor", False)
    cfg.setdefault("sae_lens_training_version", None)
    cfg.setdefault("activation_fn", "relu")
    cfg.setdefault("architecture", "standard")
    cfg.setdefault("neuronpedia_id", None)
    cfg.setdefault("reshape_activations", "hook_z" if "hook_z" in (cfg.get("hook_name") or "") else "none")
    kwargs = cfg.get("activation_fn_kwargs") or {}
    if cfg.get("activation_fn") == "topk" and kwargs.get("k") is not None:
        cfg["architecture"] = "topk"
        cfg["k"] = kwargs["k"]
    if isinstance(cfg.get("normalize_activations"), bool):
        cfg["normalize_activations"] = "expected_average_only_in" if cfg["normalize_activations"] else "none"
    if cfg.get("normalize_activations") is None:
        cfg["normalize_activations"] = "none"
    cfg.setdefault("device", "cpu")
    arch = cfg.get("architecture", "standard")
    out = filter_valid_dataclass_fields(cfg, get_sae_class(arch)[1])
    if arch == "topk" and kwargs.get("k") is not None:
        out["k"] = kwargs["k"]
    out["metadata"] = {k: v for k, v in cfg.items() if k in LLM_METADATA_KEYS}
    out["architecture"] = arch
    return out


# ------------------------------------------------------------------------------ third-party layouts
_GEMMA_WIDTHS = {"width_4k": 4096, "width_16k": 16384, "width_32k": 32768, "width_65k": 65536,
                 "width_131k": 131072, "width_262k": 262144, "width_524k": 524288, "width_1m": 1048576}
_GEMMA2_MODELS = {"2b-it": ("gemma-2-2b-it", 2304), "9b-it": ("gemma-2-9b-it", 3584),
                  "27b-it": ("gemma-2-27b-it", 4608), "2b": ("gemma-2-2b", 2304), "9b": ("gemma-2-9b", 3584),
                  "27b": ("gemma-2-27b", 4608)}


def get_gemma_2_config_from_hf(repo_id: str, folder_name: str, device: str | None,
                               force_download: bool = False,  # noqa: ARG001
                               cfg_overrides: dict[str, Any] | None = None) -> dict[str, Any]:
    d_sae = next((w for key, w in _GEMMA_WIDTHS.items() if key in folder_name), None)
    m = re.search(r"layer_(\d+)", folder_name)
    layer = int(m.group(1)) if m else (0 if "embedding" in folder_name else None)
    if layer is None:
        raise ValueError("Layer not found in folder_name and no override provided.")
    key = next((k for k in _GEMMA2_MODELS if k in repo_id), None)
    if key is None:
        raise ValueError("Model name not found in repo_id.")
    model_name, d_in = _GEMMA2_MODELS[key]
    if "res" in repo_id:
        hook = "hook_embed" if "embedding" in folder_name else f"blocks.{layer}.hook_resid_post"
    elif "mlp" in repo_id:
        hook = f"blocks.{layer}.hook_mlp_out"
    elif "att" in repo_id:
        hook = f"blocks.{layer}.attn.hook_z"
        d_in = {"2b": 2048, "9b": 4096, "27b": 4608}.get(key.split("-")[0], d_in)
    else:
        raise ValueError("Hook name not found in folder_name.")
    cfg: dict[str, Any] = {
        "architecture": "jumprelu", "d_in": d_in, "d_sae": d_sae, "dtype": "float32",
        "model_name": model_name, "hook_name": hook, "hook_head_index": None, "activation_fn": "relu",
        "finetuning_scaling_factor": False, "sae_lens_training_version": None, "prepend_bos": True,
        "dataset_path": "monology/pile-uncopyrighted", "context_size": 1024,
        "dataset_trust_remote_code": True, "apply_b_dec_to_input": False, "normalize_activations": None,
    }
    if device is not None:
        cfg["device"] = device
    if cfg_overrides:
        cfg.update(cfg_overrides)
    return cfg


def gemma_2_sae_huggingface_loader(repo_id: str, folder_name: str, device: str = "cpu",
                                   force_download: bool = False, cfg_overrides: dict[str, Any] | None = None):
    cfg = get_gemma_2_config_from_hf(repo_id, folder_name, device, force_download, cfg_overrides)
    path = _hf_download(repo_id, "params.npz", force_download, subfolder=folder_name)
    sd: dict[str, torch.Tensor] = {}
    with np.load(path) as data:
        for k in data:
            name = "W_" + k[2:] if k.startswith("w_") else k
            sd[name] = torch.tensor(data[k]).float().to(device)
    _handle_scaling_factor(cfg, sd)
    if "embedding" in folder_name:
        sd["W_enc"] = sd["W_enc"] / np.sqrt(cfg["d_in"])
        sd["W_dec"] = sd["W_dec"] * np.sqrt(cfg["d_in"])
    return cfg, sd, None


def get_llama_scope_config_from_hf(repo_id: str, folder_name: str, device: str | None,
                                   force_download: bool = False,
                                   cfg_overrides: dict[str, Any] | None = None) -> dict[str, Any]:
    with open(_hf_download(repo_id, folder_name + "/hyperparams.json", force_download)) as f:
        old = json.load(f)
    d_in = old["d_model"]
    nsf = d_in ** 0.5 / old["dataset_average_activation_norm"]["in"]
    cfg: dict[str, Any] = {
        "architecture": "jumprelu", "jump_relu_threshold": old["jump_relu_threshold"] * nsf,
        "d_in": d_in, "d_sae": old["d_sae"], "dtype": "bfloat16", "model_name": "meta-llama/Llama-3.1-8B",
        "hook_name": old["hook_point_in"], "hook_head_index": None, "activation_fn": "relu",
        "finetuning_scaling_factor": False, "sae_lens_training_version": None, "prepend_bos": True,
        "dataset_path": "cerebras/SlimPajama-627B", "context_size": 1024, "dataset_trust_remote_code": True,
        "apply_b_dec_to_input": False, "normalize_activations": "expected_average_only_in",
    }
    if device is not None:
        cfg["device"] = device
    if cfg_overrides:
        cfg.update(cfg_overrides)
    return cfg


def llama_scope_sae_huggingface_loader(repo_id: str, folder_name: str, device: str = "cpu",
                                       force_download: bool = False, cfg_overrides: dict[str, Any] | None = None):
    cfg = get_llama_scope_config_from_hf(repo_id, folder_name, device, force_download, cfg_overrides)
    path = _hf_download(repo_id, "final.safetensors", force_download, subfolder=folder_name + "/checkpoints")
    raw = load_safetensors_weights(path, device=device, dtype=cfg.get("dtype"))
    dt = str_to_dtype(cfg["dtype"])
    sd = {
        "W_enc": raw["encoder.weight"].T, "W_dec": raw["decoder.weight"].T,
        "b_enc": raw["encoder.bias"], "b_dec": raw["decoder.bias"],
        "threshold": torch.ones(cfg["d_sae"], dtype=dt, device=cfg["device"]) * cfg["jump_relu_threshold"],
    }
    return cfg, sd, None


def get_dictionary_learning_config_1_from_hf(repo_id: str, folder_name: str, device: str,
                                             force_download: bool = False,
                                             cfg_overrides: dict[str, Any] | None = None) -> dict[str, Any]:
    with open(_hf_download(repo_id, f"{folder_name}/config.json", force_download)) as f:
        config = json.load(f)
    tr, buf = config["trainer"], config["buffer"]
    act = "topk" if tr["dict_class"] == "AutoEncoderTopK" else "relu"
    arch = "standard"
    if tr["dict_class"] == "GatedAutoEncoder":
        arch = "gated"
    elif tr["dict_class"] in ("MatryoshkaBatchTopKSAE", "BatchTopKSAE"):
        arch = "jumprelu"
    cfg: dict[str, Any] = {
        "architecture": arch, "d_in": tr["activation_dim"], "d_sae": tr["dict_size"], "dtype": "float32",
        "device": device, "model_name": tr["lm_name"].split("/")[-1],
        "hook_name": f"blocks.{tr['layer']}.hook_resid_post", "hook_head_index": None,
        "activation_fn": act, "activation_fn_kwargs": {"k": tr["k"]} if act == "topk" else {},
        "apply_b_dec_to_input": True, "finetuning_scaling_factor": False, "sae_lens_training_version": None,
        "prepend_bos": True, "dataset_path": "monology/pile-uncopyrighted",
        "context_size": buf.get("ctx_len", 128), "normalize_activations": "none", "neuronpedia_id": None,
        "dataset_trust_remote_code": True,
    }
    if cfg_overrides:
        cfg.update(cfg_overrides)
    return cfg


def dictionary_learning_sae_huggingface_loader_1(repo_id: str, folder_name: str, device: str = "cpu",
                                                 force_download: bool = False,
                                                 cfg_overrides: dict[str, Any] | None = None):
    cfg = get_dictionary_learning_config_1_from_hf(repo_id, folder_name, device, force_download, cfg_overrides)
    enc = torch.load(_hf_download(repo_id, f"{folder_name}/ae.pt", force_download), map_location="cpu")
    W_enc = enc["W_enc"] if "W_enc" in enc else enc["encoder.weight"].T
    W_dec = enc["W_dec"] if "W_dec" in enc else enc["decoder.weight"].T
    sd = {"W_enc": W_enc, "W_dec": W_dec,
          "b_dec": enc.get("b_dec", enc.get("bias", enc.get("decoder_bias")))}
    for src, dst in (("encoder.bias", "b_enc"), ("b_enc", "b_enc"), ("mag_bias", "b_mag"),
                     ("gate_bias", "b_gate"), ("r_mag", "r_mag")):
        if src in enc:
            sd[dst] = enc[src]
    if "threshold" in enc:
        th = enc["threshold"]
        sd["threshold"] = torch.full((W_enc.size(1),), float(th)) if th.ndim == 0 else th
    return cfg, sd, None


def get_sparsify_config_from_disk(path: str | Path, device: str | None = None,
                                  cfg_overrides: dict[str, Any] | None = None) -> dict[str, Any]:
    path = Path(path)
    with open(path / SAE_CFG_FILENAME) as f:
        old = json.load(f)
    outer = path.parent / "config.json"
    top = json.loads(outer.read_text()) if outer.exists() else {}
    if path.name == "embed_tokens":
        hook, layer = "hook_embed", 0
    else:
        m = re.search(r"layers[._](\d+)", path.name)
        if m is None:
            raise ValueError(f"Unrecognized Sparsify folder: {path.name}")
        layer = int(m.group(1))
        hook = f"blocks.{layer}.hook_resid_post"
    d_sae = old.get("num_latents") or old["d_in"] * old["expansion_factor"]
    cfg: dict[str, Any] = {
        "architecture": "standard", "d_in": old["d_in"], "d_sae": d_sae, "dtype": "bfloat16",
        "device": device or "cpu", "model_name": top.get("model", path.parts[-2] if len(path.parts) > 1 else ""),
        "hook_name": hook, "hook_layer": layer, "hook_head_index": None, "activation_fn_str": "topk",
        "activation_fn_kwargs": {"k": old["k"], "signed": old.get("signed", False)},
        "apply_b_dec_to_input": not old.get("normalize_decoder", False),
        "dataset_path": top.get("dataset", "togethercomputer/RedPajama-Data-1T-Sample"),
        "context_size": top.get("ctx_len", 2048), "finetuning_scaling_factor": False,
        "sae_lens_training_version": None, "prepend_bos": True, "dataset_trust_remote_code": True,
        "normalize_activations": "none", "neuronpedia_id": None,
    }
    if cfg_overrides:
        cfg.update(cfg_overrides)
    return cfg


def sparsify_disk_loader(path: str | Path, device: str = "cpu",
                         cfg_overrides: dict[str, Any] | None = None) -> tuple[dict[str, Any], dict[str, torch.Tensor]]:
    cfg = get_sparsify_config_from_disk(path, device, cfg_overrides)
    raw = load_safetensors_weights(Path(path) / SPARSIFY_WEIGHTS_FILENAME, device=device, dtype=cfg.get("dtype"))
    W_enc = raw["W_enc"] if "W_enc" in raw else raw["encoder.weight"].T
    W_dec = raw["W_dec"].T if "W_dec" in raw else raw["decoder.weight"].T
    b_enc = raw["b_enc"] if "b_enc" in raw else raw["encoder.bias"]
    b_dec = raw["b_dec"] if "b_dec" in raw else raw["decoder.bias"]
    # stored decoder is [d_in, d_sae] in sparsify: transpose to [d_sae, d_in] when needed
    if W_dec.shape[0] != cfg["d_sae"]:
        W_dec = W_dec.T
    sd = {"W_enc": W_enc, "W_dec": W_dec.contiguous(), "b_enc": b_enc, "b_dec": b_dec}
    return cfg, sd


def sparsify_huggingface_loader(repo_id: str, folder_name: str, device: str = "cpu", force_download: bool = False,
                                cfg_overrides: dict[str, Any] | None = None):
    p = _hf_download(repo_id, f"{folder_name}/{SPARSIFY_WEIGHTS_FILENAME}", force_download)
    _hf_download(repo_id, f"{folder_name}/{SAE_CFG_FILENAME}", force_download)
    cfg, sd = sparsify_disk_loader(Path(p).parent, device=device, cfg_overrides=cfg_overrides)
    return cfg, sd, None


NAMED_PRETRAINED_SAE_LOADERS: dict[str, Callable[..., Any]] = {
    "sae_lens": sae_lens_huggingface_loader,
    "gemma_2": gemma_2_sae_huggingface_loader,
    "llama_scope": llama_scope_sae_huggingface_loader,
    "dictionary_learning_1": dictionary_learning_sae_huggingface_loader_1,
    "sparsify": sparsify_huggingface_loader,
}


def _register_extra_converters() -> None:
    from saelens_b200.loading import converters_extra

    NAMED_PRETRAINED_SAE_LOADERS.update(converters_extra.LOADERS)


def load_sae_config_from_huggingface(release: str, sae_id: str, device: str = "cpu",
                                     force_download: bool = False) -> dict[str, Any]:
    from saelens_b200.loading.pretrained_saes_directory import (
        get_config_overrides,
        get_conversion_loader_name,
        get_repo_id_and_folder_name,
    )

    repo_id, folder = get_repo_id_and_folder_name(release, sae_id)
    overrides = get_config_overrides(release, sae_id)
    name = get_conversion_loader_name(release)
    from saelens_b200.loading import converters_extra

    getters: dict[str, Callable[..., dict[str, Any]]] = {
        "sae_lens": get_sae_lens_config_from_hf,
        "gemma_2": get_gemma_2_config_from_hf,
        "llama_scope": get_llama_scope_config_from_hf,
        "dictionary_learning_1": get_dictionary_learning_config_1_from_hf,
        **converters_extra.CONFIG_GETTERS,
    }
    cfg = getters[name](repo_id, folder, device, force_download, overrides)
    return handle_config_defaulting(cfg)


_register_extra_converters()
