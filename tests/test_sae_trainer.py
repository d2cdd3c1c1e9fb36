"""SAETrainer step bookkeeping and logging (behaviour of sae_lens/training/sae_trainer.py; cases
follow tests/training/test_sae_trainer.py)."""

import pytest
import torch

from saelens_b200.models.sae import TrainStepOutput
from saelens_b200.models.standard import StandardTrainingSAE, StandardTrainingSAEConfig
from saelens_b200.training.sae_trainer import SAETrainer, _log_feature_sparsity, _unwrap_item
from test_training import _data, _trainer_cfg


@pytest.fixture
def trainer():
    torch.manual_seed(0)
    sae = StandardTrainingSAE(StandardTrainingSAEConfig(d_in=16, d_sae=128, l1_coefficient=2.0))
    return SAETrainer(_trainer_cfg(None, steps=20, batch=4, lr=2e-4), sae, _data(batch=4))


def test_train_step_updates_firing_statistics(trainer):
    acts = next(trainer.data_provider)
    out, _, _ = trainer._train_step(sae=trainer.sae, sae_in=acts)
    torch.testing.assert_close(out.sae_in, acts)
    assert out.sae_out.shape == acts.shape and out.feature_acts.shape == (4, 128)
    assert trainer.n_frac_active_samples == 4
    fired = (out.feature_acts > 0).float()
    torch.testing.assert_close(trainer.act_freq_scores, fired.sum(0))
    assert trainer.n_forward_passes_since_fired[fired[-1] == 1].max() == 0


def test_train_step_reduces_loss_on_repeated_input(trainer):
    acts = next(trainer.data_provider)
    first, _, _ = trainer._train_step(sae=trainer.sae, sae_in=acts)
    for _ in range(20):
        last, _, _ = trainer._train_step(sae=trainer.sae, sae_in=acts)
    assert last.loss.item() < first.loss.item()


def test_log_feature_sparsity_handles_zero():
    assert _log_feature_sparsity(torch.tensor([0.0])).item() != float("-inf")


def test_unwrap_item():
    assert _unwrap_item(3.14) == pytest.approx(3.14)
    assert _unwrap_item(torch.tensor(2.5)) == pytest.approx(2.5)
    assert _unwrap_item(lambda: torch.tensor(1.5)) == pytest.approx(1.5)
    assert _unwrap_item(lambda: 0.75) == pytest.approx(0.75)


def _output():
    return TrainStepOutput(
        sae_in=torch.tensor([[-1, 0], [0, 2], [1, 1]]).float(),
        sae_out=torch.tensor([[0, 0], [0, 2], [0.5, 1]]).float(),
        feature_acts=torch.tensor([[0, 0, 0, 1], [1, 0, 0, 1], [1, 0, 1, 1]]).float(),
        hidden_pre=torch.tensor([[-1, 0, 0, 1], [1, -1, 0, 1], [1, -1, 1, 1]]).float(),
        loss=torch.tensor(0.5), losses={"mse_loss": torch.tensor(0.25), "l1_loss": torch.tensor(0.1)},
        metrics={"topk_threshold": torch.tensor(0.5)})


@pytest.mark.parametrize("sparse", [True, False])
def test_build_train_step_log_dict(trainer, sparse):
    out = _output()
    if sparse:
        out.feature_acts = out.feature_acts.to_sparse_coo()
    d = trainer._build_train_step_log_dict(output=out, n_training_samples=123)
    want = {
        "losses/mse_loss": 0.25, "losses/l1_loss": 0.1, "losses/overall_loss": 0.5,
        "metrics/explained_variance": 0.6875, "metrics/explained_variance_legacy": 0.75,
        "metrics/explained_variance_legacy_std": 0.25, "metrics/l0": 2.0,
        "sparsity/mean_passes_since_fired": trainer.n_forward_passes_since_fired.mean().item(),
        "sparsity/dead_features": trainer.dead_neurons.sum().item(),
        "details/current_learning_rate": 2e-4, "details/l1_coefficient": 2.0, "details/n_training_samples": 123,
        "metrics/topk_threshold": 0.5,
    }
    assert d.keys() == want.keys()
    assert d == pytest.approx(want)


def test_build_train_step_log_dict_lazy_metrics(trainer):
    out = _output()
    out.metrics = {"eager": torch.tensor(1.5), "lazy_t": lambda: torch.tensor(2.5), "lazy_f": lambda: 3.5}
    d = trainer._build_train_step_log_dict(output=out, n_training_samples=100)
    assert (d["metrics/eager"], d["metrics/lazy_t"], d["metrics/lazy_f"]) == pytest.approx((1.5, 2.5, 3.5))
