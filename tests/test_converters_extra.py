"""Third-party checkpoint converters on synthetic files in each layout (hub download faked)."""

import json

import numpy as np
import pytest
import torch
import yaml
from safetensors.torch import save_file

from saelens_b200.loading import converters_extra as C
from saelens_b200.loading import pretrained_sae_loaders as base


@pytest.fixture
def hub(tmp_path, monkeypatch):
    def dl(repo_id, filename, force_download=False, subfolder=None):
        p = tmp_path / repo_id / (f"{subfolder}/{filename}" if subfolder else filename)
        if not p.exists():
            raise FileNotFoundError(str(p))
        return str(p)

    monkeypatch.setattr(base, "_hf_download", dl)

    def put(repo_id, filename, writer):
        p = tmp_path / repo_id / filename
        p.parent.mkdir(parents=True, exist_ok=True)
        writer(p)
        return p

    return put


def _lin(d_in, d_sae, enc="encoder", dec="decoder"):
    return {f"{enc}.weight": torch.randn(d_sae, d_in), f"{enc}.bias": torch.randn(d_sae),
            f"{dec}.weight": torch.randn(d_in, d_sae), f"{dec}.bias": torch.randn(d_in)}


def test_deepseek_and_goodfire(hub):
    raw = _lin(4096, 8)
    hub("ds/r1", "l19.pt", lambda p: torch.save(raw, p))
    cfg, sd, _ = C.deepseek_r1_sae_huggingface_loader("ds/r1", "l19.pt")
    assert cfg["hook_name"] == "blocks.19.hook_resid_post" and cfg["architecture"] == "standard"
    assert torch.equal(sd["W_enc"], raw["encoder.weight"].T) and sd["W_dec"].shape == (8, 4096)
    g = _lin(4096, 16, "encoder_linear", "decoder_linear")
    repo = "Goodfire/Llama-3.1-8B-Instruct-SAE-l19"
    hub(repo, "Llama-3.1-8B-Instruct-SAE-l19.pth", lambda p: torch.save(g, p))
    cfg, sd, _ = C.get_goodfire_huggingface_loader(repo, "Llama-3.1-8B-Instruct-SAE-l19.pth")
    assert cfg["hook_name"] == "blocks.19.hook_resid_post" and sd["b_dec"].shape == (4096,)
    with pytest.raises(ValueError):
        C.get_goodfire_config_from_hf("Goodfire/other", "x.pt", "cpu")


def test_llama_scope_r1_and_connor(hub):
    d_in = 32
    hub("fnlp/R1", "L5R/config.json", lambda p: p.write_text(json.dumps(
        {"d_model": d_in, "expansion_factor": 2, "hook_point_in": "blocks.5.hook_resid_post"})))
    w = {**_lin(d_in, 64), "log_jumprelu_threshold": torch.zeros(64)}
    hub("fnlp/R1", "L5R/sae_weights.safetensors", lambda p: save_file(w, str(p)))
    cfg, sd, _ = C.llama_scope_r1_distill_sae_huggingface_loader("fnlp/R1", "L5R")
    assert cfg["architecture"] == "jumprelu" and cfg["d_sae"] == 64
    assert torch.allclose(sd["threshold"], torch.ones(64))
    hub("cr/hz", "blk8_cfg.json", lambda p: p.write_text(json.dumps(
        {"act_size": 64, "dict_size": 128, "act_name": "blocks.8.attn.hook_z"})))
    hub("cr/hz", "blk8.pt", lambda p: torch.save({"W_enc": torch.randn(64, 128)}, p))
    cfg, sd, _ = C.connor_rob_hook_z_huggingface_loader("cr/hz", "blk8.pt")
    assert cfg["reshape_activations"] == "hook_z" and sd["W_enc"].shape == (64, 128)


def test_gemma_3_resid_and_transcoder(hub):
    repo = "google/gemma-scope-2-1b-pt"
    w = {"w_enc": torch.randn(16, 32), "w_dec": torch.randn(32, 16), "b_enc": torch.randn(32), "b_dec": torch.randn(16),
         "threshold": torch.rand(32)}
    hub(repo, "resid_post/layer_7_width_32/params.safetensors", lambda p: save_file(w, str(p)))
    cfg, sd, _ = C.gemma_3_sae_huggingface_loader(repo, "resid_post/layer_7_width_32")
    assert cfg["hook_name"] == "blocks.7.hook_resid_post" and cfg["architecture"] == "jumprelu"
    assert cfg["model_name"] == "google/gemma-3-1b-pt" and cfg["d_in"] == 16 and cfg["d_sae"] == 32
    wt = {**w, "affine_skip_connection": torch.randn(16, 16)}
    hub(repo, "transcoder_affine/layer_3_width_32/params.safetensors", lambda p: save_file(wt, str(p)))
    cfg, sd, _ = C.gemma_3_sae_huggingface_loader(repo, "transcoder_affine/layer_3_width_32")
    assert cfg["architecture"] == "jumprelu_skip_transcoder" and cfg["hook_name_out"] == "blocks.3.hook_mlp_out"
    assert "W_skip" in sd and cfg["d_out"] == 16


def test_gemma_2_transcoder_mwhanna_mntss_temporal(hub):
    repo = "google/gemma-scope-2b-pt-transcoders"
    arrs = {"W_enc": np.random.randn(2304, 16).astype(np.float32), "W_dec": np.random.randn(16, 2304).astype(np.float32),
            "b_enc": np.zeros(16, np.float32), "b_dec": np.zeros(2304, np.float32), "threshold": np.ones(16, np.float32)}
    hub(repo, "layer_3/width_16k/canonical/params.npz", lambda p: np.savez(p, **arrs))
    cfg, sd, _ = C.gemma_2_transcoder_huggingface_loader(repo, "layer_3/width_16k/canonical")
    assert cfg["d_sae"] == 16384 and cfg["model_name"] == "gemma-2-2b" and sd["threshold"].shape == (16,)
    mw = "mwhanna/qwen3-0.6b-transcoders"
    hub(mw, "wandb-config.yaml", lambda p: p.write_text(yaml.safe_dump(
        {"d_model": {"value": 32}, "d_feature": {"value": 64}, "batch_size": {"value": 128}})))
    hub(mw, "layer_2.safetensors", lambda p: save_file({"W_enc": torch.randn(64, 32), "W_dec": torch.randn(64, 32),
                                                         "b_enc": torch.zeros(64), "b_dec": torch.zeros(32)}, str(p)))
    cfg, sd, _ = C.mwhanna_transcoder_huggingface_loader(mw, "layer_2.safetensors")
    assert cfg["model_name"] == "Qwen/Qwen3-0.6B" and sd["W_enc"].shape == (32, 64)
    mn = "mntss/clt"
    hub(mn, "config.yaml", lambda p: p.write_text(yaml.safe_dump(
        {"model_name": "gpt2", "feature_input_hook": "hook_resid_mid", "feature_output_hook": "hook_mlp_out"})))
    hub(mn, "W_enc_1.safetensors", lambda p: save_file({"W_enc_1": torch.randn(64, 32), "b_enc_1": torch.zeros(64),
                                                         "b_dec_1": torch.zeros(32)}, str(p)))
    hub(mn, "W_dec_1.safetensors", lambda p: save_file({"W_dec_1": torch.randn(64, 3, 32)}, str(p)))
    with pytest.warns(UserWarning):
        cfg, sd, _ = C.mntss_clt_layer_huggingface_loader(mn, "1")
    assert cfg["d_sae"] == 64 and sd["W_dec"].shape == (64, 32) and cfg["hook_name"] == "blocks.1.hook_resid_mid"
    tp = "canrager/temporalSAEs"
    hub(tp, "gemma_layer_12/conf.yaml", lambda p: p.write_text(yaml.safe_dump(
        {"llm": {"dimin": 16}, "data": {"dtype": "float32"},
         "sae": {"exp_factor": 2, "n_heads": 2, "n_attn_layers": 1, "bottleneck_factor": 1, "sae_diff_type": "topk",
                 "kval_topk": 4, "tied_weights": False, "scaling_factor": 1.5}})))
    hub(tp, "gemma_layer_12/latest_ckpt.safetensors", lambda p: save_file(
        {"D": torch.randn(32, 16), "b": torch.zeros(16), "E": torch.randn(16, 32),
         "attn_layers.0.q.weight": torch.randn(4, 4)}, str(p)))
    cfg, sd, _ = C.temporal_sae_huggingface_loader(tp, "gemma_layer_12")
    assert cfg["d_sae"] == 32 and cfg["hook_name"] == "blocks.12.hook_resid_post"
    assert set(sd) == {"W_dec", "b_dec", "W_enc", "attn_layers.0.q.weight"}


def test_all_fourteen_registered():
    assert set(base.NAMED_PRETRAINED_SAE_LOADERS) == {
        "sae_lens", "connor_rob_hook_z", "gemma_2", "gemma_3", "llama_scope", "llama_scope_r1_distill",
        "dictionary_learning_1", "deepseek_r1", "sparsify", "gemma_2_transcoder", "mwhanna_transcoder",
        "mntss_clt_layer_transcoder", "temporal", "goodfire"}
