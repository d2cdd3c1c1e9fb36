"""Further third-party SAE / transcoder checkpoint converters (the remaining layouts of
sae_lens/loading/pretrained_sae_loaders.py:1886-1901): connor_rob_hook_z, gemma_3, llama_scope_r1_distill,
deepseek_r1, gemma_2_transcoder, mwhanna_transcoder, mntss_clt_layer_transcoder, temporal, goodfire.

Each loader takes `(repo_id, folder_name, device, force_download, cfg_overrides)` and returns
`(cfg_dict, state_dict, None)` with the native weight names (W_enc [d_in, d_sae], W_dec [d_sae,
d_out], b_enc, b_dec, threshold, W_skip, ...).  Files come through `_hf_download`; shapes that the
reference reads from the hub's safetensors header are read from the downloaded file instead.
"""

from __future__ import annotations

import json
import re
import warnings
from typing import Any

import numpy as np
import torch

from saelens_b200.utils.misc import str_to_dtype


def _dl(repo_id: str, filename: str, force_download: bool = False, subfolder: str | None = None) -> str:
    from saelens_b200.loading import pretrained_sae_loaders as base  # the registry imports this module

    return base._hf_download(repo_id, filename, force_download, subfolder)


def _missing() -> tuple[type[BaseException], ...]:
    from saelens_b200.loading import pretrained_sae_loaders as base

    return base.MISSING_FILE_ERRORS


def _load_st(path: str, device: str = "cpu", dtype: Any = None) -> dict[str, torch.Tensor]:
    from saelens_b200.loading import pretrained_sae_loaders as base

    return base.load_safetensors_weights(path, device=device, dtype=dtype)


def _yaml(path: str) -> dict[str, Any]:
    import yaml

    with open(path) as f:
        return yaml.safe_load(f)


def _layer(text: str, pattern: str = r"layer_(\d+)") -> int:
    m = re.search(pattern, text)
    if m is None:
        raise ValueError(f"could not find a layer index in {text!r}")
    return int(m.group(1))


def _shapes(path: str) -> dict[str, list[int]]:
    """Tensor shapes from a safetensors file's JSON header."""
    with open(path, "rb") as f:
        n = int.from_bytes(f.read(8), "little")
        meta = json.loads(f.read(n))
    return {k: v["shape"] for k, v in meta.items() if k != "__metadata__"}


def _merge(cfg: dict[str, Any], device: str | None, overrides: dict[str, Any] | None) -> dict[str, Any]:
    cfg["device"] = device if device is not None else "cpu"
    cfg.update(overrides or {})
    return cfg


# ------------------------------------------------------------------------------ connor_rob_hook_z
def get_connor_rob_hook_z_config_from_hf(repo_id: str, folder_name: str, device: str | None = None,
                                         force_download: bool = False,
                                         cfg_overrides: dict[str, Any] | None = None) -> dict[str, Any]:
    raw = json.load(open(_dl(repo_id, folder_name.split(".pt")[0] + "_cfg.json", force_download)))
    return _merge({"architecture": "standard", "d_in": raw["act_size"], "d_sae": raw["dict_size"], "dtype": "float32",
                   "model_name": "gpt2-small", "hook_name": raw["act_name"], "hook_head_index": None,
                   "activation_fn": "relu", "apply_b_dec_to_input": True, "finetuning_scaling_factor": False,
                   "sae_lens_training_version": None, "prepend_bos": True, "dataset_path": "Skylion007/openwebtext",
                   "context_size": 128, "normalize_activations": "none", "reshape_activations": "hook_z"},
                  device, cfg_overrides)


def connor_rob_hook_z_huggingface_loader(repo_id: str, folder_name: str, device: str = "cpu",
                                         force_download: bool = False, cfg_overrides: dict[str, Any] | None = None):
    cfg = get_connor_rob_hook_z_config_from_hf(repo_id, folder_name, device, force_download, cfg_overrides)
    sd = torch.load(_dl(repo_id, folder_name, force_download), map_location=device)
    return cfg, dict(sd), None


# ------------------------------------------------------------------------------ deepseek_r1
def get_deepseek_r1_config_from_hf(repo_id: str, folder_name: str, device: str, force_download: bool = False,
                                   cfg_overrides: dict[str, Any] | None = None) -> dict[str, Any]:
    layer = _layer(folder_name, r"l(\d+)")
    return _merge({"architecture": "standard", "d_in": 4096, "d_sae": 4096 * 16, "dtype": "bfloat16",
                   "context_size": 1024, "model_name": "deepseek-ai/DeepSeek-R1-Distill-Llama-8B",
                   "hook_name": f"blocks.{layer}.hook_resid_post", "hook_head_index": None, "prepend_bos": True,
                   "dataset_path": "lmsys/lmsys-chat-1m", "sae_lens_training_version": None,
                   "activation_fn": "relu", "normalize_activations": "none", "apply_b_dec_to_input": False,
                   "finetuning_scaling_factor": False}, device, cfg_overrides)


def _linear_pair(sd: dict[str, torch.Tensor], enc: str, dec: str) -> dict[str, torch.Tensor]:
    return {"W_enc": sd[f"{enc}.weight"].T, "W_dec": sd[f"{dec}.weight"].T, "b_enc": sd[f"{enc}.bias"],
            "b_dec": sd[f"{dec}.bias"]}


def deepseek_r1_sae_huggingface_loader(repo_id: str, folder_name: str, device: str = "cpu",
                                       force_download: bool = False, cfg_overrides: dict[str, Any] | None = None):
    cfg = get_deepseek_r1_config_from_hf(repo_id, folder_name, device, force_download, cfg_overrides)
    raw = torch.load(_dl(repo_id, folder_name, force_download), map_location=device)
    return cfg, _linear_pair(raw, "encoder", "decoder"), None


# ------------------------------------------------------------------------------ llama_scope_r1_distill
def get_llama_scope_r1_distill_config_from_hf(repo_id: str, folder_name: str, device: str,
                                              force_download: bool = False,
                                              cfg_overrides: dict[str, Any] | None = None) -> dict[str, Any]:
    raw = json.load(open(_dl(repo_id, folder_name + "/config.json", force_download)))
    d_in = raw["d_model"]
    return _merge({"architecture": "jumprelu", "d_in": d_in, "d_sae": d_in * raw["expansion_factor"],
                   "dtype": "float32", "model_name": "meta-llama/Llama-3.1-8B", "hook_name": raw["hook_point_in"],
                   "hook_head_index": None, "activation_fn": "relu", "finetuning_scaling_factor": False,
                   "sae_lens_training_version": None, "prepend_bos": True, "dataset_path": "cerebras/SlimPajama-627B",
                   "context_size": 1024, "apply_b_dec_to_input": False,
                   "normalize_activations": "expected_average_only_in"}, device, cfg_overrides)


def llama_scope_r1_distill_sae_huggingface_loader(repo_id: str, folder_name: str, device: str = "cpu",
                                                  force_download: bool = False,
                                                  cfg_overrides: dict[str, Any] | None = None):
    cfg = get_llama_scope_r1_distill_config_from_hf(repo_id, folder_name, device, force_download, cfg_overrides)
    raw = _load_st(_dl(repo_id, "sae_weights.safetensors", force_download, folder_name),
                                        device=device, dtype=cfg.get("dtype"))
    sd = _linear_pair(raw, "encoder", "decoder")
    sd["threshold"] = raw["log_jumprelu_threshold"].exp()
    return cfg, sd, None


# ------------------------------------------------------------------------------ gemma_3
def _gemma_3_hooks(repo_id: str, folder_name: str) -> dict[str, Any]:
    layer = _layer(folder_name)
    tc = "transcoder" in folder_name or "clt" in folder_name
    if tc:
        hin, hout = f"model.layers.{layer}.pre_feedforward_layernorm.output", \
            f"model.layers.{layer}.post_feedforward_layernorm.output"
    elif "resid_post" in folder_name:
        hin, hout = f"model.layers.{layer}.output", None
    elif "attn_out" in folder_name:
        hin, hout = f"model.layers.{layer}.self_attn.o_proj.input", None
    elif "mlp_out" in folder_name:
        hin, hout = f"model.layers.{layer}.post_feedforward_layernorm.output", None
    else:
        raise ValueError(f"could not infer the hook type of {folder_name!r}")
    raw: dict[str, Any] = {"architecture": "jump_relu", "model_name": repo_id.replace("gemma-scope-2", "gemma-3"),
                           "hf_hook_point_in": hin}
    if tc:
        raw["affine_connection"] = "affine" in folder_name
    if hout:
        raw["hf_hook_point_out"] = hout
    return raw


def _gemma_3_params_path(repo_id: str, folder_name: str, force_download: bool) -> str:
    if "clt" in folder_name:
        sub, fname = "/".join(folder_name.split("/")[:-1]), folder_name.split("/")[-1] + ".safetensors"
        return _dl(repo_id, fname, force_download, sub or None)
    return _dl(repo_id, "params.safetensors", force_download, folder_name)


def get_gemma_3_config_from_hf(repo_id: str, folder_name: str, device: str, force_download: bool = False,
                               cfg_overrides: dict[str, Any] | None = None) -> dict[str, Any]:
    try:
        raw = json.load(open(_dl(repo_id, f"{folder_name}/config.json", force_download)))
    except Exception:  # no config in the repo: infer from the names
        raw = _gemma_3_hooks(repo_id, folder_name)
    if raw.get("architecture") != "jump_relu":
        raise ValueError(f"unexpected Gemma 3 architecture {raw.get('architecture')!r}")
    layer = _layer(folder_name)
    tc = "transcoder" in folder_name or "clt" in folder_name
    if "resid_post" in folder_name:
        hook, hook_out = f"blocks.{layer}.hook_resid_post", None
    elif "attn_out" in folder_name:
        hook, hook_out = f"blocks.{layer}.attn.hook_z", None
    elif "mlp_out" in folder_name:
        hook, hook_out = f"blocks.{layer}.hook_mlp_out", None
    elif tc:
        hook, hook_out = f"blocks.{layer}.hook_mlp_in", f"blocks.{layer}.hook_mlp_out"
    else:
        raise ValueError("hook name not found in folder_name")
    shapes = _shapes(_gemma_3_params_path(repo_id, folder_name, force_download))
    d_in, d_sae = shapes["w_enc"]
    model = raw["model_name"]
    model = (model if "google" in model else "google/" + model).replace("-v3", "-3")
    if "270m" in model:
        model = model.replace("-pt", "")
    arch = "jumprelu"
    if tc:
        arch = "jumprelu_skip_transcoder" if raw.get("affine_connection", False) else "jumprelu_transcoder"
    cfg = {"architecture": arch, "d_in": d_in, "d_sae": d_sae, "dtype": "float32", "model_name": model,
           "hook_name": hook, "hook_head_index": None, "finetuning_scaling_factor": False,
           "sae_lens_training_version": None, "prepend_bos": True, "dataset_path": "monology/pile-uncopyrighted",
           "context_size": 1024, "apply_b_dec_to_input": False, "normalize_activations": "none",
           "reshape_activations": "none", "hf_hook_name": raw.get("hf_hook_point_in")}
    if hook_out:
        cfg["hook_name_out"] = hook_out
        cfg["hf_hook_name_out"] = raw.get("hf_hook_point_out")
        cfg["d_out"] = shapes["w_dec"][-1]
    return _merge(cfg, device, cfg_overrides)


def gemma_3_sae_huggingface_loader(repo_id: str, folder_name: str, device: str = "cpu", force_download: bool = False,
                                   cfg_overrides: dict[str, Any] | None = None):
    cfg = get_gemma_3_config_from_hf(repo_id, folder_name, device, force_download, cfg_overrides)
    raw = _load_st(_gemma_3_params_path(repo_id, folder_name, force_download), device=device,
                                        dtype=cfg.get("dtype"))
    w_dec = raw["w_dec"].sum(dim=1).contiguous() if "clt" in folder_name else raw["w_dec"]
    sd = {"W_enc": raw["w_enc"], "W_dec": w_dec, "b_enc": raw["b_enc"], "b_dec": raw["b_dec"],
          "threshold": raw["threshold"]}
    if "affine_skip_connection" in raw:
        sd["W_skip"] = raw["affine_skip_connection"]
    return cfg, sd, None


# ------------------------------------------------------------------------------ gemma_2_transcoder
_GEMMA_WIDTHS = {"width_4k": 4096, "width_16k": 16384, "width_65k": 65536, "width_262k": 262144,
                 "width_524k": 524288, "width_1m": 1048576}
_GEMMA_MODELS = [("2b-it", "gemma-2-2b-it", 2304), ("2b", "gemma-2-2b", 2304), ("9b-it", "gemma-2-9b-it", 3584),
                 ("9b", "gemma-2-9b", 3584), ("27b-it", "gemma-2-27b-it", 4608), ("27b", "gemma-2-27b", 4608)]


def get_gemma_2_transcoder_config_from_hf(repo_id: str, folder_name: str, device: str | None = None,
                                          force_download: bool = False,
                                          cfg_overrides: dict[str, Any] | None = None) -> dict[str, Any]:
    d_sae = next((v for k, v in _GEMMA_WIDTHS.items() if k in folder_name), None)
    if d_sae is None:
        m = re.search(r"width_(\d+)k", folder_name)
        if m is None:
            raise ValueError(f"could not find the dictionary size in {folder_name!r}")
        d_sae = int(m.group(1)) * 1024
    try:
        layer = _layer(folder_name)
    except ValueError:
        layer = _layer(repo_id)
    found = next(((name, dim) for key, name, dim in _GEMMA_MODELS if key in repo_id), None)
    if found is None:
        raise ValueError(f"could not determine the model from {repo_id!r}")
    name, dim = found
    return _merge({"architecture": "jumprelu_transcoder", "d_in": dim, "d_out": dim, "d_sae": d_sae,
                   "dtype": "float32", "activation_fn": "relu", "normalize_activations": "none", "model_name": name,
                   "hook_name": f"blocks.{layer}.ln2.hook_normalized", "hook_name_out": f"blocks.{layer}.hook_mlp_out",
                   "hook_head_index": None, "hook_head_index_out": None, "prepend_bos": True,
                   "dataset_path": "monology/pile-uncopyrighted", "context_size": 1024,
                   "apply_b_dec_to_input": False}, device, cfg_overrides)


def gemma_2_transcoder_huggingface_loader(repo_id: str, folder_name: str, device: str = "cpu",
                                          force_download: bool = False, cfg_overrides: dict[str, Any] | None = None):
    cfg = get_gemma_2_transcoder_config_from_hf(repo_id, folder_name, device, force_download, cfg_overrides)
    params = np.load(_dl(repo_id, f"{folder_name}/params.npz", force_download))
    names = {"w_enc": "W_enc", "wenc": "W_enc", "w_e": "W_enc", "w_dec": "W_dec", "wdec": "W_dec", "w_d": "W_dec",
             "b_enc": "b_enc", "benc": "b_enc", "b_e": "b_enc", "b_dec": "b_dec", "bdec": "b_dec", "b_d": "b_dec",
             "threshold": "threshold"}
    sd = {names[k.lower()]: torch.tensor(params[k], dtype=torch.float32, device=device)
          for k in params.files if k.lower() in names}
    return cfg, sd, None


# ------------------------------------------------------------------------------ mwhanna_transcoder
def get_mwhanna_transcoder_config_from_hf(repo_id: str, folder_name: str, device: str | None = None,
                                          force_download: bool = False,
                                          cfg_overrides: dict[str, Any] | None = None) -> dict[str, Any]:
    layer = int(folder_name.replace(".safetensors", "").split("_")[-1])
    try:
        wb = _yaml(_dl(repo_id, "wandb-config.yaml", force_download))
    except _missing():
        wb = _yaml(_dl(repo_id, "wanb-config.yaml", force_download))
    try:
        base_cfg = _yaml(_dl(repo_id, "config.yaml", force_download))
    except _missing():
        m = re.search(r"qwen3-(\d+(?:\.\d+)?)b", repo_id)
        if m is None:
            raise ValueError(f"could not find the Qwen3 size in {repo_id!r}") from None
        base_cfg = {"model_name": f"Qwen/Qwen3-{m.group(1)}B"}
    return _merge({"architecture": "transcoder", "d_in": wb["d_model"]["value"], "d_out": wb["d_model"]["value"],
                   "d_sae": wb["d_feature"]["value"], "dtype": "float32", "activation_fn": "relu",
                   "normalize_activations": "none", "model_name": base_cfg["model_name"],
                   "hook_name": f"blocks.{layer}.mlp.hook_in", "hook_name_out": f"blocks.{layer}.hook_mlp_out",
                   "dataset_path": "monology/pile-uncopyrighted", "context_size": wb["batch_size"]["value"],
                   "apply_b_dec_to_input": False, "model_from_pretrained_kwargs": {"fold_ln": False}},
                  device, cfg_overrides)


def mwhanna_transcoder_huggingface_loader(repo_id: str, folder_name: str, device: str = "cpu",
                                          force_download: bool = False, cfg_overrides: dict[str, Any] | None = None):
    cfg = get_mwhanna_transcoder_config_from_hf(repo_id, folder_name, device, force_download, cfg_overrides)
    sd = _load_st(_dl(repo_id, folder_name, force_download), device=device, dtype=cfg.get("dtype"))
    sd["W_enc"] = sd["W_enc"].T
    return cfg, sd, None


# ------------------------------------------------------------------------------ mntss_clt_layer_transcoder
def get_mntss_clt_layer_config_from_hf(repo_id: str, folder_name: str, device: str, force_download: bool = False,
                                       cfg_overrides: dict[str, Any] | None = None) -> dict[str, Any]:
    info = _yaml(_dl(repo_id, "config.yaml", force_download))
    shapes = _shapes(_dl(repo_id, f"W_enc_{folder_name}.safetensors", force_download))
    d = shapes[f"b_dec_{folder_name}"][0]
    return _merge({"architecture": "transcoder", "d_in": d, "d_out": d, "d_sae": shapes[f"b_enc_{folder_name}"][0],
                   "dtype": "float32", "activation_fn": "relu", "normalize_activations": "none",
                   "model_name": info["model_name"], "hook_name": f"blocks.{folder_name}.{info['feature_input_hook']}",
                   "hook_name_out": f"blocks.{folder_name}.{info['feature_output_hook']}",
                   "apply_b_dec_to_input": False, "model_from_pretrained_kwargs": {"fold_ln": False}},
                  device, cfg_overrides)


def mntss_clt_layer_huggingface_loader(repo_id: str, folder_name: str, device: str = "cpu",
                                       force_download: bool = False, cfg_overrides: dict[str, Any] | None = None):
    """One layer of a cross-layer transcoder as a single-layer transcoder: the decoders to every
    later layer are summed, so use it to read feature activations, not for reconstruction."""
    warnings.warn("loading a CLT layer with summed decoders: for feature activations, not reconstruction",
                  UserWarning, stacklevel=2)
    cfg = get_mntss_clt_layer_config_from_hf(repo_id, folder_name, device, force_download, cfg_overrides)
    enc = _load_st(_dl(repo_id, f"W_enc_{folder_name}.safetensors", force_download),
                                        device=device, dtype=cfg.get("dtype"))
    dec = _load_st(_dl(repo_id, f"W_dec_{folder_name}.safetensors", force_download),
                                        device=device, dtype=cfg.get("dtype"))
    sd = {"W_enc": enc[f"W_enc_{folder_name}"].T, "b_enc": enc[f"b_enc_{folder_name}"],
          "b_dec": enc[f"b_dec_{folder_name}"], "W_dec": dec[f"W_dec_{folder_name}"].sum(dim=1)}
    return cfg, sd, None


# ------------------------------------------------------------------------------ temporal
def get_temporal_sae_config_from_hf(repo_id: str, folder_name: str, device: str, force_download: bool = False,
                                    cfg_overrides: dict[str, Any] | None = None) -> dict[str, Any]:
    y = _yaml(_dl(repo_id, f"{folder_name}/conf.yaml", force_download))
    d_in = y["llm"]["dimin"]
    s = y["sae"]
    cfg = {"architecture": "temporal", "hook_name": f"blocks.{_layer(folder_name)}.hook_resid_post", "d_in": d_in,
           "d_sae": int(d_in * s["exp_factor"]), "n_heads": s["n_heads"], "n_attn_layers": s["n_attn_layers"],
           "bottleneck_factor": s["bottleneck_factor"], "sae_diff_type": s["sae_diff_type"],
           "kval_topk": s["kval_topk"], "tied_weights": s["tied_weights"], "dtype": y["data"]["dtype"],
           "normalize_activations": "constant_scalar_rescale",
           "activation_normalization_factor": s["scaling_factor"], "apply_b_dec_to_input": True}
    return _merge(cfg, device, cfg_overrides)


def temporal_sae_huggingface_loader(repo_id: str, folder_name: str, device: str = "cpu", force_download: bool = False,
                                    cfg_overrides: dict[str, Any] | None = None):
    cfg = get_temporal_sae_config_from_hf(repo_id, folder_name, device, force_download, cfg_overrides)
    raw = _load_st(_dl(repo_id, f"{folder_name}/latest_ckpt.safetensors", force_download),
                                        device=device, dtype=cfg.get("dtype"))
    sd = {k: v for k, v in raw.items() if k.startswith("attn_layers.")}
    sd["W_dec"] = raw["D"]
    sd["b_dec"] = raw["b"]
    if "E" in raw:
        sd["W_enc"] = raw["E"]
    return cfg, sd, None


# ------------------------------------------------------------------------------ goodfire
_GOODFIRE = {
    ("Goodfire/Llama-3.3-70B-Instruct-SAE-l50", "Llama-3.3-70B-Instruct-SAE-l50.pt"):
        (8192, 65536, "meta-llama/Llama-3.3-70B-Instruct", 50),
    ("Goodfire/Llama-3.1-8B-Instruct-SAE-l19", "Llama-3.1-8B-Instruct-SAE-l19.pth"):
        (4096, 65536, "meta-llama/Llama-3.1-8B-Instruct", 19),
}


def get_goodfire_config_from_hf(repo_id: str, folder_name: str, device: str, force_download: bool = False,
                                cfg_overrides: dict[str, Any] | None = None) -> dict[str, Any]:
    if (repo_id, folder_name) not in _GOODFIRE:
        raise ValueError(f"unsupported Goodfire SAE: {repo_id}/{folder_name}")
    d_in, d_sae, model, layer = _GOODFIRE[(repo_id, folder_name)]
    return _merge({"architecture": "standard", "d_in": d_in, "d_sae": d_sae, "model_name": model,
                   "hook_name": f"blocks.{layer}.hook_resid_post", "hook_head_index": None,
                   "dataset_path": "lmsys/lmsys-chat-1m", "apply_b_dec_to_input": False}, device, cfg_overrides)


def get_goodfire_huggingface_loader(repo_id: str, folder_name: str, device: str = "cpu", force_download: bool = False,
                                    cfg_overrides: dict[str, Any] | None = None):
    cfg = get_goodfire_config_from_hf(repo_id, folder_name, device, force_download, cfg_overrides)
    raw = torch.load(_dl(repo_id, folder_name, force_download), map_location=device)
    dt = str_to_dtype(cfg.get("dtype", "float32"))
    sd = {k: v.to(dt) for k, v in _linear_pair(raw, "encoder_linear", "decoder_linear").items()}
    return cfg, sd, None


LOADERS = {
    "connor_rob_hook_z": connor_rob_hook_z_huggingface_loader,
    "gemma_3": gemma_3_sae_huggingface_loader,
    "llama_scope_r1_distill": llama_scope_r1_distill_sae_huggingface_loader,
    "deepseek_r1": deepseek_r1_sae_huggingface_loader,
    "gemma_2_transcoder": gemma_2_transcoder_huggingface_loader,
    "mwhanna_transcoder": mwhanna_transcoder_huggingface_loader,
    "mntss_clt_layer_transcoder": mntss_clt_layer_huggingface_loader,
    "temporal": temporal_sae_huggingface_loader,
    "goodfire": get_goodfire_huggingface_loader,
}
CONFIG_GETTERS = {
    "connor_rob_hook_z": get_connor_rob_hook_z_config_from_hf,
    "gemma_3": get_gemma_3_config_from_hf,
    "llama_scope_r1_distill": get_llama_scope_r1_distill_config_from_hf,
    "deepseek_r1": get_deepseek_r1_config_from_hf,
    "gemma_2_transcoder": get_gemma_2_transcoder_config_from_hf,
    "mwhanna_transcoder": get_mwhanna_transcoder_config_from_hf,
    "mntss_clt_layer_transcoder": get_mntss_clt_layer_config_from_hf,
    "temporal": get_temporal_sae_config_from_hf,
    "goodfire": get_goodfire_config_from_hf,
}
