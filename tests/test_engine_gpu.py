"""The fused native TopK training step against a plain PyTorch fp32 restatement."""

import math

import pytest
import torch

pytestmark = pytest.mark.gpu


def _setup(d_in=256, d_sae=2048, k=32, B=512, seed=0, b_dec_scale=0.05):
    from saelens_b200.models.topk import TopKTrainingSAE, TopKTrainingSAEConfig

    torch.manual_seed(seed)
    sae = TopKTrainingSAE(TopKTrainingSAEConfig(d_in=d_in, d_sae=d_sae, k=k, device="cuda"))
    with torch.no_grad():
        sae.b_enc.normal_(0, 0.01)
        sae.b_dec.normal_(0, b_dec_scale)
        sae.W_enc.add_(torch.randn_like(sae.W_enc) * 0.01)
    x = torch.randn(B, d_in, device="cuda")
    return sae, x


def _oracle(w_enc_bf16, w_dec_bf16, b_enc, b_dec, x_bf16, idx, k):
    """fp32 autograd of the reference TopK training loss for a given per-row selection."""
    We = w_enc_bf16.float().T.clone().requires_grad_(True)  # [d_in, d_sae]
    Wd = w_dec_bf16.float().clone().requires_grad_(True)
    be = b_enc.float().clone().requires_grad_(True)
    bd = b_dec.float().clone().requires_grad_(True)
    x = x_bf16.float()
    sae_in = x - bd
    pre = sae_in @ We + be
    norm = Wd.norm(dim=-1)
    h = pre * norm
    sel = torch.gather(h, 1, idx.long())
    acts = torch.zeros_like(h).scatter(1, idx.long(), sel.relu())
    out = (acts / norm) @ Wd + bd
    mse = (out - x).pow(2).sum(-1).mean()
    mse.backward()
    return mse.detach(), h.detach(), {"W_enc": We.grad, "W_dec": Wd.grad, "b_enc": be.grad, "b_dec": bd.grad}


def _rel(a, b):
    return ((a.float() - b.float()).norm() / (b.float().norm() + 1e-12)).item()


@pytest.mark.parametrize("b_enc_shift", [0.0, -0.25])
def test_engine_gradients_match_fp32_autograd(b_enc_shift):
    """b_enc_shift < 0 makes about half of the selected pre-activations negative: those pairs are
    not live (ReLU zero) and must drop out of the gradient pair lists."""
    from saelens_b200.training.engine import FusedTopKEngine

    sae, x = _setup()
    with torch.no_grad():
        sae.b_enc.add_(b_enc_shift)
    eng = FusedTopKEngine(sae, lr=1e-3)
    xb = x.to(torch.bfloat16)
    w_enc0, w_dec0 = eng.w_enc.clone(), eng.w_dec.clone()
    b_enc0, b_dec0 = eng.p_benc.clone(), eng.p_bdec.clone()
    res = eng.step(xb, update=False)
    torch.cuda.synchronize()
    eng.status.check()
    mse, h, grads = _oracle(w_enc0, w_dec0, b_enc0, b_dec0, xb, res.topk_idx, eng.k)
    # selection is a valid top-k of the fp32 pre-activations up to bf16 rounding of H
    kth = torch.topk(h, eng.k, dim=-1).values[:, -1:]
    chosen = torch.gather(h, 1, res.topk_idx.long())
    assert (chosen >= kth - 0.02 * kth.abs() - 1e-3).all()
    assert abs(res.mse_loss.item() - mse.item()) <= 2e-2 * mse.item()
    # gradient rows are written only for latents with a live pair (Adam skips the others by
    # colptr); the oracle's gradient must vanish on those rows
    live = (eng.colptr[1:] > eng.colptr[:-1])
    assert live.any()
    assert grads["W_dec"][~live].abs().max().item() == 0.0 if (~live).any() else True
    assert _rel(eng.g_dec[live], grads["W_dec"][live]) < 2e-2
    assert _rel(eng.g_enc[live], grads["W_enc"].T[live]) < 2e-2
    assert _rel(eng.g_benc, grads["b_enc"]) < 2e-2


def test_engine_adam_step_matches_torch_adam():
    from saelens_b200.training.engine import FusedTopKEngine

    sae, x = _setup(seed=1)
    eng = FusedTopKEngine(sae, lr=1e-3)
    xb = x.to(torch.bfloat16)
    w_enc0, w_dec0 = eng.w_enc.clone(), eng.w_dec.clone()
    b_enc0, b_dec0 = eng.p_benc.clone(), eng.p_bdec.clone()
    p_enc0, p_dec0 = eng.p_enc.clone(), eng.p_dec.clone()
    res = eng.step(xb, update=True)
    torch.cuda.synchronize()
    _, _, grads = _oracle(w_enc0, w_dec0, b_enc0, b_dec0, xb, res.topk_idx, eng.k)
    # torch reference: clip_grad_norm_(1.0) then one Adam step from the same fp32 masters
    params = {"W_enc": p_enc0.T.clone(), "W_dec": p_dec0.clone(), "b_enc": b_enc0.clone(), "b_dec": b_dec0.clone()}
    ps = [torch.nn.Parameter(v.clone()) for v in params.values()]
    for p, name in zip(ps, params):
        p.grad = grads[name].float().clone()
    total = torch.nn.utils.clip_grad_norm_(ps, 1.0)
    assert abs(eng.grad_norm().item() - total.item()) <= 2e-2 * total.item()
    opt = torch.optim.Adam(ps, lr=1e-3)
    opt.step()
    # first Adam step moves every parameter with a non-negligible gradient by ~lr
    for p, name, got in zip(ps, params, [eng.p_enc.T, eng.p_dec, eng.p_benc, eng.p_bdec]):
        d_ref = p.detach() - params[name]
        d_got = got - params[name]
        big = grads[name].abs() > 1e-3 * grads[name].abs().max()
        agree = (torch.sign(d_ref[big]) == torch.sign(d_got[big])).float().mean().item()
        assert agree > 0.99, (name, agree)
        assert torch.allclose(d_got[big], d_ref[big], atol=2e-4, rtol=0.05), name


def test_engine_training_reduces_loss_and_tracks_stats():
    from saelens_b200.training.engine import FusedTopKEngine

    sae, x = _setup(d_in=512, d_sae=4096, k=32, B=1024, seed=2)
    eng = FusedTopKEngine(sae, lr=2e-3)
    xb = x.to(torch.bfloat16)
    act = torch.zeros(4096, device="cuda")
    since = torch.zeros(4096, device="cuda")
    losses = [eng.step(xb, act_freq=act, since_fired=since).loss.item() for _ in range(30)]
    torch.cuda.synchronize()
    eng.status.check()
    assert all(math.isfinite(v) for v in losses)
    assert losses[-1] < 0.7 * losses[0]
    assert int(act.sum().item()) > 0
    assert ((since == 0) == (eng.fire_counts > 0)).all()


def test_engine_aux_loss_matches_reference():
    from saelens_b200.training.engine import FusedTopKEngine

    sae, x = _setup(d_in=256, d_sae=1024, k=16, B=256, seed=3)
    import copy

    ref_sae = copy.deepcopy(sae)
    eng = FusedTopKEngine(sae, lr=1e-3)
    xb = x.to(torch.bfloat16)
    dead = torch.zeros(1024, dtype=torch.bool, device="cuda")
    dead[::3] = True
    res = eng.step(xb, dead_mask=dead, run_aux=True, update=False)
    torch.cuda.synchronize()
    eng.status.check()
    # reference aux loss from the module math with bf16-rounded weights
    with torch.no_grad():
        ref_sae.W_enc.copy_(eng.w_enc.float().T)
        ref_sae.W_dec.copy_(eng.w_dec.float())
        ref_sae.b_dec.copy_(eng.p_bdec)
        ref_sae.b_enc.copy_(eng.p_benc)
    from saelens_b200.models.sae import TrainStepInput

    out = ref_sae.training_forward_pass(TrainStepInput(sae_in=xb.float(), coefficients={}, dead_neuron_mask=dead))
    ref_aux = out.losses["auxiliary_reconstruction_loss"].item()
    assert ref_aux > 0
    assert abs(res.aux_loss.item() - ref_aux) <= 5e-2 * ref_aux


def test_batchtopk_engine_selection_and_gradients():
    """BatchTopK on the fused engine: exactly k*B activations are kept batch-wide (the largest ReLU
    values up to bf16 ties), rows keep variable counts, gradients match fp32 autograd on the
    engine's selection, and the threshold EMA moves toward the smallest kept activation."""
    from saelens_b200.models.batchtopk import BatchTopKTrainingSAE, BatchTopKTrainingSAEConfig
    from saelens_b200.training.engine import FusedTopKEngine

    torch.manual_seed(0)
    sae = BatchTopKTrainingSAE(BatchTopKTrainingSAEConfig(d_in=256, d_sae=2048, k=16, device="cuda"))
    with torch.no_grad():
        sae.b_enc.normal_(0, 0.01)
        sae.b_dec.normal_(0, 0.05)
    x = torch.randn(512, 256, device="cuda").to(torch.bfloat16)
    eng = FusedTopKEngine(sae, lr=1e-3)
    w_enc0, w_dec0 = eng.w_enc.clone(), eng.w_dec.clone()
    b_enc0, b_dec0 = eng.p_benc.clone(), eng.p_bdec.clone()
    res = eng.step(x, update=False)
    torch.cuda.synchronize()
    eng.status.check()
    sel = res.topk_idx >= 0
    K = 16 * 512
    assert int(sel.sum()) == K
    per_row = sel.sum(1)
    assert per_row.max() > per_row.min()  # a batch-wide, not per-row, selection
    assert int(eng.batch_truncated.item()) == 0
    # oracle pre-activations (fp32 of the bf16 compute copies)
    We, Wd = w_enc0.float().T, w_dec0.float()
    norm = Wd.norm(dim=-1)
    h = ((x.float() - b_dec0) @ We + b_enc0) * norm
    kth = torch.topk(h.relu().flatten(), K).values[-1]
    chosen = torch.gather(h, 1, res.topk_idx.clamp(min=0).long())[sel]
    assert (chosen >= kth - 0.02 * kth.abs() - 1e-3).all()
    # gradients against fp32 autograd with the engine's selection as the mask
    mask = torch.zeros_like(h, dtype=torch.bool)
    rows = torch.arange(512, device="cuda")[:, None].expand_as(res.topk_idx)
    mask[rows[sel], res.topk_idx[sel].long()] = True
    Wd_ = Wd.clone().requires_grad_(True)
    We_ = We.clone().requires_grad_(True)
    be = b_enc0.clone().requires_grad_(True)
    bd = b_dec0.clone().requires_grad_(True)
    n_ = Wd_.norm(dim=-1)
    hh = ((x.float() - bd) @ We_ + be) * n_
    acts = torch.where(mask, hh.relu(), torch.zeros_like(hh))
    out = (acts / n_) @ Wd_ + bd
    mse = (out - x.float()).pow(2).sum(-1).mean()
    mse.backward()
    assert abs(res.mse_loss.item() - mse.item()) <= 2e-2 * mse.item()
    live = (eng.colptr[1:] > eng.colptr[:-1])
    assert _rel(eng.g_dec[live], Wd_.grad[live]) < 2e-2
    assert _rel(eng.g_enc[live], We_.grad.T[live]) < 2e-2
    # threshold EMA: 0.99 * 0 + 0.01 * (smallest kept activation)
    kept_min = res.topk_vals[sel].min().double()
    assert torch.allclose(sae.topk_threshold, 0.01 * kept_min, rtol=1e-5)


def test_matryoshka_engine_nested_losses_and_gradients():
    """Matryoshka BatchTopK on the native engine: the nested prefix MSEs and every gradient against
    fp32 autograd of sum_l MSE(prefix_l reconstruction) with the engine's selection as the mask."""
    from saelens_b200.models.batchtopk import MatryoshkaBatchTopKTrainingSAE, MatryoshkaBatchTopKTrainingSAEConfig
    from saelens_b200.training.matryoshka_engine import MatryoshkaEngine, matryoshka_engine_supported

    torch.manual_seed(0)
    widths = [256, 768, 2048]
    sae = MatryoshkaBatchTopKTrainingSAE(MatryoshkaBatchTopKTrainingSAEConfig(
        d_in=256, d_sae=2048, k=16, matryoshka_widths=list(widths), device="cuda"))
    with torch.no_grad():
        sae.b_enc.normal_(0, 0.01)
        sae.b_dec.normal_(0, 0.05)
    assert matryoshka_engine_supported(sae)
    x = torch.randn(512, 256, device="cuda").to(torch.bfloat16)
    eng = MatryoshkaEngine(sae, lr=1e-3)
    w_enc0, w_dec0 = eng.w_enc.clone(), eng.w_dec.clone()
    b_enc0, b_dec0 = eng.p_benc.clone(), eng.p_bdec.clone()
    res = eng.step(x, update=False)
    torch.cuda.synchronize()
    eng.status.check()
    sel = res.topk_idx >= 0
    mask = torch.zeros(512, 2048, dtype=torch.bool, device="cuda")
    rows = torch.arange(512, device="cuda")[:, None].expand_as(res.topk_idx)
    mask[rows[sel], res.topk_idx[sel].long()] = True
    We = w_enc0.float().T.clone().requires_grad_(True)
    Wd = w_dec0.float().clone().requires_grad_(True)
    be = b_enc0.clone().requires_grad_(True)
    bd = b_dec0.clone().requires_grad_(True)
    n_ = Wd.norm(dim=-1)
    hh = ((x.float() - bd) @ We + be) * n_
    acts = torch.where(mask, hh.relu(), torch.zeros_like(hh)) / n_
    total = 0.0
    mses = []
    for w in widths:
        rec = acts[:, :w] @ Wd[:w] + bd
        m = (rec - x.float()).pow(2).sum(-1).mean()
        mses.append(m)
        total = total + m
    total.backward()
    assert abs(res.mse_loss.item() - mses[-1].item()) <= 1e-2 * mses[-1].item()
    for w, m in zip(widths[:-1], mses[:-1]):
        got = res.extra_losses[f"inner_mse_loss_{w}"].item()
        assert abs(got - m.item()) <= 1e-2 * m.item(), (w, got, m.item())
    live = eng.colptr[1:] > eng.colptr[:-1]

    def rel(a, b):
        return ((a.float() - b.float()).norm() / b.float().norm()).item()

    assert rel(eng.g_dec[live], Wd.grad[live]) < 3e-2
    assert rel(eng.g_enc[live], We.grad.T[live]) < 3e-2
    assert rel(eng.g_benc[live], be.grad[live]) < 3e-2
    losses = [float(eng.step(x).loss) for _ in range(5)]
    assert losses[-1] < losses[0]
