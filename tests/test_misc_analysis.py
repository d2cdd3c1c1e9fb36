"""Results report, Neuronpedia URL/request building, HF upload (fake API), TSEA and the HF bridge."""

import json
import types

import pytest
import torch

from saelens_b200.analysis import neuronpedia as npd
from saelens_b200.analysis.results import build_report, format_report
from saelens_b200.analysis.tsea import calculate_batch_enrichment_scores, get_test_gene_sets, pad_gene_sets


def _run(root, ts, samples, elapsed, steps, cfg=None, hooks=None):
    d = root / f"saelens_runner_gpu_{ts}"
    d.mkdir()
    with open(d / "timing_history.jsonl", "w") as f:
        for i in range(steps):
            f.write(json.dumps({"step": i + 1, "n_training_samples": samples * (i + 1) // steps,
                                "elapsed_s": elapsed * (i + 1) / steps}) + "\n")
    if cfg is not None:
        (d / "runner_cfg.json").write_text(json.dumps(cfg))
    for h in hooks or []:
        (d / f"blocks_{h}").mkdir()


def test_results_report(tmp_path):
    _run(tmp_path, "250101_000001", 1000, 10.0, 40, {"hook_name": "a", "training_tokens": 1000})
    _run(tmp_path, "250101_000002", 500, 10.0, 40, {"hook_name": "a", "training_tokens": 500})
    _run(tmp_path, "250101_000003", 100, 10.0, 5, {"hook_name": "a", "training_tokens": 1000})
    _run(tmp_path, "250101_000004", 800, 4.0, 40, None, hooks=[1, 2])
    rep = build_report(tmp_path)
    assert sorted(rep.groups) == [1, 2]
    g1 = rep.groups[1].rows
    assert [r.scenario for r in g1] == ["baseline", "vDP+sDP(fsdp)", "sDP(fsdp)+bs8"]
    assert g1[0].local_tokens_per_s == pytest.approx(100.0)
    assert g1[1].normalized_tokens_per_s == pytest.approx(100.0)  # 500 tokens scaled to the 1000 budget
    assert not g1[2].complete and "short_steps" in g1[2].notes and "under_target_tokens" in g1[2].notes
    assert rep.groups[1].best_complete.run_id.endswith("000001")
    assert "missing_cfg" in rep.groups[2].rows[0].notes
    assert "baseline" in format_report(rep)


def test_neuronpedia_urls_and_bodies():
    meta = types.SimpleNamespace(neuronpedia_id="gpt2-small/0-res-jb", model_name="gpt2-small")
    sae = types.SimpleNamespace(cfg=types.SimpleNamespace(metadata=meta))
    assert npd.open_neuronpedia_feature_dashboard(sae, 5, open_browser=False) == "https://neuronpedia.org/gpt2-small/0-res-jb/5"
    url = npd.get_neuronpedia_quick_list(sae, [1, 2], name="my list", open_browser=False)
    assert url.startswith("https://neuronpedia.org/quick-list/?name=my%20list&features=")
    assert npd.feature_api_url(3, 7) == "https://neuronpedia.org/api/feature/gpt2-small/7-res-jb/3"
    body = npd.list_request_body("l", [npd.NeuronpediaFeature("gpt2-small", 0, "res-jb", 9, "d")])
    assert body["features"][0]["layer"] == "0-res-jb"
    assert json.loads('[Infinity, -Infinity, NaN]', parse_constant=npd.NanAndInfReplacer) == [9999, -9999, 0]
    assert npd.sanitize_for_json({"a": [float("inf"), 1.0]}) == {"a": [9999, 1.0]}
    f = npd.NeuronpediaFeature("m", 0, "d", 1, activations=[npd.NeuronpediaActivation("x", ["a"], [0.5])])
    assert f.has_activating_text()
    bad = types.SimpleNamespace(cfg=types.SimpleNamespace(metadata=types.SimpleNamespace(neuronpedia_id=None)))
    with pytest.raises(ValueError):
        npd.feature_dashboard_url(bad, 1)


class _FakeApi:
    def __init__(self):
        self.calls = []

    def create_repo(self, repo_id, exist_ok=True):
        self.calls.append(("create", repo_id))

    def upload_folder(self, folder_path, path_in_repo, **kw):
        import os

        self.calls.append(("folder", path_in_repo, sorted(os.listdir(folder_path))))

    def file_exists(self, repo_id, filename, revision=None):
        return False

    def upload_file(self, path_or_fileobj, path_in_repo, **kw):
        self.calls.append(("file", path_in_repo, path_or_fileobj.read().decode()))


def test_upload_saes_with_fake_api(tmp_path):
    from saelens_b200.models.standard import StandardSAE, StandardSAEConfig
    from saelens_b200.training.upload_saes_to_huggingface import upload_saes_to_huggingface

    sae = StandardSAE(StandardSAEConfig(d_in=8, d_sae=16))
    sae.save_model(str(tmp_path / "saved"))
    api = _FakeApi()
    upload_saes_to_huggingface({"a": sae, "b": str(tmp_path / "saved")}, "me/repo", show_progress=False, api=api)
    folders = [c for c in api.calls if c[0] == "folder"]
    assert [c[1] for c in folders] == ["a", "b"] and "cfg.json" in folders[0][2]
    readme = [c for c in api.calls if c[0] == "file"][0][2]
    assert "- a" in readme and "me/repo" in readme
    with pytest.raises(FileNotFoundError):
        upload_saes_to_huggingface({"x": str(tmp_path / "missing")}, "me/repo", api=api)


def test_tsea_enrichment():
    V = 10
    scores = torch.tensor([[9.0, 8, 7, 6, 5, 4, 3, 2, 1, 0], [0, 1, 2, 3, 4, 5, 6, 7, 8, 9]])
    sets = pad_gene_sets({"top": {0, 1, 2}, "mid": {4, 5}})
    es = calculate_batch_enrichment_scores(scores, torch.tensor(list(sets.values())))
    assert es[0, 0] == pytest.approx(1.0)  # the set sits at the top of feature 0's ranking
    assert es[0, 1] == pytest.approx(1.0)  # and at the bottom of feature 1's (|running sum| reaches 1)
    assert es[1, 0] < es[0, 0]
    vocab = {"Ġthe": 0, "The": 1, "123": 2, ",": 3, "Ġred": 4}
    gs = get_test_gene_sets(vocab)
    assert gs["starts_with_space"] == {0, 4} and gs["all_digits"] == {2} and gs["colors"] == {4}
    _ = V


def test_bridge_boots_hf_model_and_splices_sae():
    transformers = pytest.importorskip("transformers")
    from saelens_b200.analysis.sae_transformer_bridge import SAETransformerBridge
    from saelens_b200.models.standard import StandardSAE, StandardSAEConfig

    cfg = transformers.GPT2Config(n_layer=2, n_embd=32, n_head=4, vocab_size=100, n_positions=32)
    torch.manual_seed(0)
    hf = transformers.GPT2LMHeadModel(cfg).eval()
    br = SAETransformerBridge.boot_transformers(hf, dtype="float32")
    toks = torch.randint(0, 100, (2, 8))
    with torch.no_grad():
        ref = hf(toks).logits
        out = br(toks)
    assert torch.allclose(out, ref, atol=1e-4)
    sae = StandardSAE(StandardSAEConfig(d_in=32, d_sae=64))
    sae.cfg.metadata.hook_name = "blocks.0.hook_resid_post"
    with torch.no_grad():
        spliced = br.run_with_saes(toks, saes=[sae], use_error_term=True)
    assert torch.allclose(spliced, ref, atol=1e-3)  # error term restores the clean activations
    assert br.acts_to_saes == {}


def test_hook_name_layer_helpers_and_temporary_seed():
    from saelens_b200.utils.misc import (
        extract_layer_from_tlens_hook_name,
        extract_stop_at_layer_from_tlens_hook_name,
        temporary_seed,
    )

    assert extract_layer_from_tlens_hook_name("blocks.12.hook_resid_pre") == 12
    assert extract_layer_from_tlens_hook_name("blocks.3.attn.hook_z") == 3
    assert extract_layer_from_tlens_hook_name("hook_embed") is None
    assert extract_stop_at_layer_from_tlens_hook_name("blocks.12.hook_resid_pre") == 13
    assert extract_stop_at_layer_from_tlens_hook_name("ln_final.hook_normalized") is None
    torch.manual_seed(0)
    before = torch.random.get_rng_state()
    with temporary_seed(123):
        a = torch.rand(3)
    with temporary_seed(123):
        b = torch.rand(3)
    assert torch.equal(a, b) and torch.equal(torch.random.get_rng_state(), before)
