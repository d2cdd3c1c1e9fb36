"""CPU tests of the SAE zoo: encode/decode math, losses, folding, save/load round trips."""

import math

import pytest
import torch

from saelens_b200 import (
    SAE,
    BatchTopKTrainingSAE,
    BatchTopKTrainingSAEConfig,
    GatedSAE,
    GatedSAEConfig,
    GatedTrainingSAE,
    GatedTrainingSAEConfig,
    JumpReLUSAE,
    JumpReLUSAEConfig,
    JumpReLUTrainingSAE,
    JumpReLUTrainingSAEConfig,
    MatchingPursuitSAE,
    MatchingPursuitSAEConfig,
    MatchingPursuitTrainingSAE,
    MatchingPursuitTrainingSAEConfig,
    MatryoshkaBatchTopKTrainingSAE,
    MatryoshkaBatchTopKTrainingSAEConfig,
    SkipTranscoder,
    SkipTranscoderConfig,
    StandardSAE,
    StandardSAEConfig,
    StandardTrainingSAE,
    StandardTrainingSAEConfig,
    TemporalSAE,
    TemporalSAEConfig,
    TopKSAE,
    TopKSAEConfig,
    TopKTrainingSAE,
    TopKTrainingSAEConfig,
    TrainingSAE,
    Transcoder,
    TranscoderConfig,
    TrainStepInput,
)


def _step_input(x, dead=None, coeffs=None):
    return TrainStepInput(sae_in=x, coefficients=coeffs or {}, dead_neuron_mask=dead)


def test_standard_encode_decode_math():
    sae = StandardSAE(StandardSAEConfig(d_in=8, d_sae=16))
    with torch.no_grad():
        sae.b_dec.normal_()
        sae.b_enc.normal_()
    x = torch.randn(5, 8)
    f = sae.encode(x)
    assert torch.allclose(f, torch.relu((x - sae.b_dec) @ sae.W_enc + sae.b_enc))
    assert torch.allclose(sae.decode(f), f @ sae.W_dec + sae.b_dec)
    assert torch.allclose(sae(x), sae.decode(f))


def test_training_init_tied_and_norm():
    sae = StandardTrainingSAE(StandardTrainingSAEConfig(d_in=8, d_sae=32, decoder_init_norm=0.1))
    assert torch.allclose(sae.W_dec.norm(dim=-1), torch.full((32,), 0.1), atol=1e-6)
    assert torch.allclose(sae.W_enc, sae.W_dec.T)


def test_standard_l1_loss_matches_formula():
    sae = StandardTrainingSAE(StandardTrainingSAEConfig(d_in=8, d_sae=16, l1_coefficient=5.0))
    x = torch.randn(7, 8)
    out = sae.training_forward_pass(_step_input(x, coeffs={"l1": 5.0}))
    f = out.feature_acts
    l1 = (5.0 * (f * sae.W_dec.norm(dim=1)).norm(p=1, dim=-1)).mean()
    mse = (out.sae_out - x).pow(2).sum(-1).mean()
    assert torch.allclose(out.losses["l1_loss"], l1)
    assert torch.allclose(out.losses["mse_loss"], mse)
    assert torch.allclose(out.loss, l1 + mse)


def test_topk_keeps_k_and_relu():
    sae = TopKSAE(TopKSAEConfig(d_in=8, d_sae=32, k=4))
    f = sae.encode(torch.randn(6, 8))
    assert ((f != 0).sum(-1) <= 4).all()
    assert (f >= 0).all()


def test_topk_training_rescale_matches_manual():
    sae = TopKTrainingSAE(TopKTrainingSAEConfig(d_in=8, d_sae=32, k=4))
    with torch.no_grad():
        sae.W_dec.mul_(torch.rand(32, 1) + 0.5)
    x = torch.randn(6, 8)
    acts, pre = sae.encode_with_hidden_pre(x)
    n = sae.W_dec.norm(dim=-1)
    ref_pre = ((x - sae.b_dec) @ sae.W_enc + sae.b_enc) * n
    assert torch.allclose(pre, ref_pre, atol=1e-6)
    v, i = ref_pre.topk(4, dim=-1)
    ref_acts = torch.zeros_like(ref_pre).scatter(-1, i, v.relu())
    assert torch.allclose(acts, ref_acts, atol=1e-6)
    out = sae.decode(acts)
    assert torch.allclose(out, (acts / n) @ sae.W_dec + sae.b_dec, atol=1e-5)


def test_topk_aux_loss_zero_without_dead_and_positive_with_dead():
    sae = TopKTrainingSAE(TopKTrainingSAEConfig(d_in=8, d_sae=32, k=4))
    x = torch.randn(16, 8)
    out = sae.training_forward_pass(_step_input(x, dead=torch.zeros(32, dtype=torch.bool)))
    assert out.losses["auxiliary_reconstruction_loss"].item() == 0.0
    dead = torch.zeros(32, dtype=torch.bool)
    dead[:10] = True
    out = sae.training_forward_pass(_step_input(x, dead=dead))
    assert out.losses["auxiliary_reconstruction_loss"].item() > 0


def test_topk_sparse_activations_match_dense():
    cfg = dict(d_in=8, d_sae=32, k=4)
    dense = TopKTrainingSAE(TopKTrainingSAEConfig(**cfg))
    sparse = TopKTrainingSAE(TopKTrainingSAEConfig(**cfg, use_sparse_activations=True))
    sparse.load_state_dict(dense.state_dict())
    x = torch.randn(5, 8)
    a = dense.training_forward_pass(_step_input(x))
    b = sparse.training_forward_pass(_step_input(x))
    assert torch.allclose(a.sae_out, b.sae_out, atol=1e-5)


def test_topk_fold_and_inference_export(tmp_path):
    sae = TopKTrainingSAE(TopKTrainingSAEConfig(d_in=8, d_sae=32, k=4))
    with torch.no_grad():
        sae.W_dec.mul_(torch.rand(32, 1) + 0.5)
        sae.b_enc.normal_()
    x = torch.randn(5, 8)
    before = sae(x)
    sae.save_inference_model(tmp_path)
    inf = SAE.load_from_disk(tmp_path)
    assert isinstance(inf, TopKSAE)
    assert torch.allclose(inf.W_dec.norm(dim=-1), torch.ones(32), atol=1e-5)
    assert torch.allclose(inf(x), before, atol=1e-4)


def test_batchtopk_average_k_and_jumprelu_export(tmp_path):
    sae = BatchTopKTrainingSAE(BatchTopKTrainingSAEConfig(d_in=8, d_sae=64, k=3))
    x = torch.randn(20, 8)
    out = sae.training_forward_pass(_step_input(x))
    assert (out.feature_acts > 0).sum().item() <= 3 * 20
    assert out.metrics["topk_threshold"].dtype == torch.float64
    assert sae.topk_threshold.item() > 0
    sae.save_inference_model(tmp_path)
    inf = SAE.load_from_disk(tmp_path)
    assert isinstance(inf, JumpReLUSAE)
    assert torch.allclose(inf.threshold, torch.full((64,), float(sae.topk_threshold)), atol=1e-5)


def test_matryoshka_inner_losses():
    with pytest.warns(UserWarning):
        sae = MatryoshkaBatchTopKTrainingSAE(
            MatryoshkaBatchTopKTrainingSAEConfig(d_in=8, d_sae=32, k=4, matryoshka_widths=[8, 16])
        )
    assert sae.cfg.matryoshka_widths == [8, 16, 32]
    out = sae.training_forward_pass(_step_input(torch.randn(10, 8)))
    assert "inner_mse_loss_8" in out.losses and "inner_mse_loss_16" in out.losses
    with pytest.raises(ValueError):
        MatryoshkaBatchTopKTrainingSAE(MatryoshkaBatchTopKTrainingSAEConfig(d_in=8, d_sae=32, k=4,
                                                                            matryoshka_widths=[16, 8, 32]))


def test_jumprelu_threshold_grads_and_roundtrip(tmp_path):
    sae = JumpReLUTrainingSAE(JumpReLUTrainingSAEConfig(d_in=8, d_sae=16, jumprelu_init_threshold=0.01))
    x = torch.randn(32, 8)
    out = sae.training_forward_pass(_step_input(x, coeffs={"l0": 1.0}))
    out.loss.backward()
    assert sae.log_threshold.grad is not None
    sae.save_model(tmp_path)
    from safetensors.torch import load_file

    sd = load_file(tmp_path / "sae_weights.safetensors")
    assert "threshold" in sd and "log_threshold" not in sd
    assert torch.allclose(sd["threshold"], torch.exp(sae.log_threshold.detach()))
    loaded = TrainingSAE.load_from_disk(tmp_path)
    assert torch.allclose(loaded.log_threshold, sae.log_threshold, atol=1e-6)


def test_jumprelu_tanh_mode_and_pre_act_loss():
    sae = JumpReLUTrainingSAE(JumpReLUTrainingSAEConfig(d_in=8, d_sae=16, jumprelu_sparsity_loss_mode="tanh",
                                                        pre_act_loss_coefficient=3e-6))
    dead = torch.ones(16, dtype=torch.bool)
    out = sae.training_forward_pass(_step_input(torch.randn(4, 8), dead=dead, coeffs={"l0": 1.0}))
    assert "pre_act_loss" in out.losses


def test_jumprelu_inference_fold_keeps_outputs():
    sae = JumpReLUSAE(JumpReLUSAEConfig(d_in=8, d_sae=16))
    with torch.no_grad():
        sae.W_dec.mul_(torch.rand(16, 1) + 0.5)
        sae.threshold.fill_(0.05)
        sae.b_enc.normal_()
    x = torch.randn(5, 8)
    before = sae(x)
    sae.fold_W_dec_norm()
    assert torch.allclose(sae(x), before, atol=1e-5)


def test_gated_losses_and_fold():
    sae = GatedTrainingSAE(GatedTrainingSAEConfig(d_in=8, d_sae=16))
    with torch.no_grad():
        sae.r_mag.normal_(0, 0.1)
        sae.b_gate.normal_(0, 0.1)
    x = torch.randn(9, 8)
    out = sae.training_forward_pass(_step_input(x, coeffs={"l1": 1.0}))
    assert set(out.losses) == {"mse_loss", "l1_loss", "auxiliary_reconstruction_loss"}
    inf = GatedSAE(GatedSAEConfig(d_in=8, d_sae=16))
    inf.load_state_dict(sae.state_dict())
    with torch.no_grad():
        inf.W_dec.mul_(torch.rand(16, 1) + 0.5)
    before = inf(x)
    inf.fold_W_dec_norm()
    assert torch.allclose(inf(x), before, atol=1e-5)
    with pytest.raises(ValueError):
        GatedTrainingSAE(GatedTrainingSAEConfig(d_in=8, d_sae=16), use_error_term=True)


def test_transcoders():
    tc = Transcoder(TranscoderConfig(d_in=8, d_sae=16, d_out=4, apply_b_dec_to_input=False))
    x = torch.randn(3, 8)
    y, acts = tc.forward_with_activations(x)
    assert y.shape == (3, 4) and acts.shape == (3, 16)
    sk = SkipTranscoder(SkipTranscoderConfig(d_in=8, d_sae=16, d_out=4, apply_b_dec_to_input=False))
    with torch.no_grad():
        sk.W_skip.normal_()
    assert torch.allclose(sk(x), sk.decode(sk.encode(x)) + x @ sk.W_skip.T)
    with pytest.raises(ValueError):
        TranscoderConfig(d_in=8, d_sae=16, d_out=4)


def test_temporal_sae_shapes_and_causality():
    sae = TemporalSAE(TemporalSAEConfig(d_in=16, d_sae=64, n_heads=2, bottleneck_factor=8, kval_topk=4))
    x = torch.randn(2, 5, 16)
    y = sae(x)
    assert y.shape == x.shape
    x2 = x.clone()
    x2[:, -1] += 10.0
    z1, p1 = sae.encode_with_predictions(x)
    z2, p2 = sae.encode_with_predictions(x2)
    assert torch.allclose(p1[:, :-1], p2[:, :-1], atol=1e-5)  # predictions never look ahead


def test_matching_pursuit_reconstructs_tied():
    sae = MatchingPursuitSAE(MatchingPursuitSAEConfig(d_in=8, d_sae=32, residual_threshold=1e-3))
    with torch.no_grad():
        sae.W_dec.copy_(torch.nn.functional.normalize(torch.randn(32, 8), dim=-1))
    assert torch.equal(sae.W_enc, sae.W_dec.T)
    x = sae.W_dec[3] * 2.0 + sae.b_dec
    acts = sae.encode(x.unsqueeze(0))
    assert acts[0, 3].item() == pytest.approx(2.0, rel=1e-4)
    tr = MatchingPursuitTrainingSAE(MatchingPursuitTrainingSAEConfig(d_in=8, d_sae=32, decoder_init_norm=1.0))
    out = tr.training_forward_pass(TrainStepInput(sae_in=torch.randn(4, 8), coefficients={},
                                                  dead_neuron_mask=None, is_logging_step=True))
    assert "residual_norm" in out.metrics


@pytest.mark.parametrize("arch_cls,cfg_cls,extra", [
    (StandardTrainingSAE, StandardTrainingSAEConfig, {}),
    (TopKTrainingSAE, TopKTrainingSAEConfig, {"k": 4}),
    (GatedTrainingSAE, GatedTrainingSAEConfig, {}),
    (JumpReLUTrainingSAE, JumpReLUTrainingSAEConfig, {}),
])
def test_training_save_load_roundtrip(tmp_path, arch_cls, cfg_cls, extra):
    sae = arch_cls(cfg_cls(d_in=8, d_sae=16, **extra))
    sae.save_model(tmp_path)
    loaded = TrainingSAE.load_from_disk(tmp_path)
    assert type(loaded) is arch_cls
    for k, v in sae.state_dict().items():
        assert torch.allclose(loaded.state_dict()[k], v, atol=1e-6), k


def test_error_term_reconstructs_input_exactly():
    sae = StandardSAE(StandardSAEConfig(d_in=8, d_sae=16))
    x = torch.randn(4, 8)
    with pytest.warns(DeprecationWarning):
        sae.use_error_term = True
    assert torch.allclose(sae(x), x, atol=1e-5)


def test_normalization_modes_roundtrip():
    for mode in ("constant_norm_rescale", "layer_norm"):
        sae = StandardSAE(StandardSAEConfig(d_in=8, d_sae=16, normalize_activations=mode))
        x = torch.randn(3, 8) * 7 + 2
        f = sae.encode(x)
        out = sae.decode(f)
        assert out.shape == x.shape and math.isfinite(out.sum().item())
    with pytest.raises(ValueError):
        StandardSAEConfig(d_in=8, d_sae=16, normalize_activations="bogus")  # type: ignore[arg-type]


def test_fold_activation_norm_scaling_factor():
    sae = StandardSAE(StandardSAEConfig(d_in=8, d_sae=16))
    x = torch.randn(5, 8)
    sf = 3.0
    before = sae(x * sf) / sf
    sae.fold_activation_norm_scaling_factor(sf)
    assert torch.allclose(sae(x), before, atol=1e-5)
