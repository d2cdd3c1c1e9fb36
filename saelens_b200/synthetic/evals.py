"""Metrics for SAEs trained on synthetic data with known ground-truth features (role of
sae_lens/synthetic/evals.py): decoder/feature alignment (MCC with an optimal one-to-one matching,
uniqueness), per-latent classification of the matched feature's firing, L0, dead latents,
shrinkage and explained variance."""

from __future__ import annotations

from dataclasses import asdict, dataclass
from typing import Any

import torch

from saelens_b200.utils.misc import cosine_similarities


def mean_correlation_coefficient(features_a: torch.Tensor, features_b: torch.Tensor) -> float:
    """Mean |cos| over the one-to-one matching that maximises it (Hungarian algorithm); see O'Neill et
    al., arXiv:2411.13117."""
    from scipy.optimize import linear_sum_assignment

    sim = cosine_similarities(features_a.float(), features_b.float()).abs()
    r, c = linear_sum_assignment(-sim.cpu().numpy())
    return float(sim[torch.as_tensor(r), torch.as_tensor(c)].mean())


def feature_uniqueness(sae_features: torch.Tensor, gt_features: torch.Tensor) -> float:
    """Distinct best-matching ground-truth features / number of SAE latents."""
    if sae_features.shape[0] == 0:
        return 0.0
    best = cosine_similarities(sae_features.float(), gt_features.float()).abs().argmax(dim=1)
    return best.unique().numel() / sae_features.shape[0]


@dataclass
class ClassificationMetrics:
    precision: float
    recall: float
    f1_score: float
    accuracy: float


class ClassificationMetricsCalculator:
    """Each latent, as a detector of its best-matching ground-truth feature (by decoder cosine),
    accumulates TP/FP/FN/TN over batches; metrics are means over latents."""

    def __init__(self, sae_decoder: torch.Tensor, gt_features: torch.Tensor):
        self.n = sae_decoder.shape[0]
        self.best = (cosine_similarities(sae_decoder.float(), gt_features.float()).abs().argmax(dim=1)
                     if self.n else torch.empty(0, dtype=torch.long))
        self.counts = torch.zeros(4, self.n, dtype=torch.float64)

    def add_batch(self, sae_latents: torch.Tensor, gt_feature_acts: torch.Tensor) -> None:
        if self.n == 0:
            return
        s = sae_latents > 0
        g = gt_feature_acts.to_dense()[:, self.best.to(gt_feature_acts.device)] > 0 if gt_feature_acts.is_sparse \
            else gt_feature_acts[:, self.best.to(gt_feature_acts.device)] > 0
        self.counts += torch.stack([(s & g).sum(0), (s & ~g).sum(0), (~s & g).sum(0), (~s & ~g).sum(0)]).double().cpu()

    def compute(self) -> ClassificationMetrics:
        if self.n == 0:
            return ClassificationMetrics(0.0, 0.0, 0.0, 0.0)
        tp, fp, fn, tn = self.counts

        def ratio(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
            return torch.where(b > 0, a / b.clamp(min=1e-12), torch.zeros_like(a))

        prec, rec = ratio(tp, tp + fp), ratio(tp, tp + fn)
        f1 = ratio(2 * prec * rec, prec + rec)
        acc = ratio(tp + tn, tp + fp + fn + tn)
        return ClassificationMetrics(float(prec.mean()), float(rec.mean()), float(f1.mean()), float(acc.mean()))


def compute_classification_metrics(sae_latents: torch.Tensor, gt_feature_acts: torch.Tensor,
                                   sae_decoder: torch.Tensor, gt_features: torch.Tensor) -> ClassificationMetrics:
    c = ClassificationMetricsCalculator(sae_decoder, gt_features)
    c.add_batch(sae_latents, gt_feature_acts)
    return c.compute()


class L0Calculator:
    def __init__(self) -> None:
        self.total = 0.0
        self.rows = 0

    def add_batch(self, activations: torch.Tensor) -> None:
        if activations.is_sparse:
            self.total += float((activations.coalesce().values() != 0).sum())
        else:
            self.total += float((activations != 0).sum())
        self.rows += activations.shape[0]

    def compute(self) -> float:
        return self.total / max(self.rows, 1)


class DeadLatentsCalculator:
    def __init__(self, num_latents: int) -> None:
        self.fired = torch.zeros(num_latents, dtype=torch.bool)

    def add_batch(self, sae_latents: torch.Tensor) -> None:
        self.fired |= (sae_latents != 0).any(dim=0).cpu()

    def compute(self) -> int:
        return int((~self.fired).sum())


class ShrinkageCalculator:
    """Mean of ||sae_output|| / ||input|| over samples whose input norm exceeds min_input_norm."""

    def __init__(self, min_input_norm: float = 1e-6) -> None:
        self.min_input_norm = min_input_norm
        self.total = 0.0
        self.n = 0

    def add_batch(self, sae_output: torch.Tensor, hidden_acts: torch.Tensor) -> None:
        n_in = hidden_acts.float().norm(dim=-1)
        ok = n_in > self.min_input_norm
        self.total += float((sae_output.float().norm(dim=-1)[ok] / n_in[ok]).sum())
        self.n += int(ok.sum())

    def compute(self) -> float:
        return self.total / max(self.n, 1)


class ExplainedVarianceCalculator:
    """1 - sum ||x - x_hat||^2 / sum ||x - mean(x)||^2, streaming (per-dimension sums)."""

    def __init__(self, hidden_dim: int, device: torch.device | str = "cpu") -> None:
        self.sum_x = torch.zeros(hidden_dim, dtype=torch.float64, device=device)
        self.sum_x2 = torch.zeros((), dtype=torch.float64, device=device)
        self.sum_err = torch.zeros((), dtype=torch.float64, device=device)
        self.n = 0

    def add_batch(self, sae_output: torch.Tensor, hidden_acts: torch.Tensor) -> None:
        x = hidden_acts.double().to(self.sum_x.device)
        self.sum_x += x.sum(0)
        self.sum_x2 += x.square().sum()
        self.sum_err += (x - sae_output.double().to(x.device)).square().sum()
        self.n += x.shape[0]

    def compute(self) -> float:
        if self.n == 0:
            return 0.0
        total = self.sum_x2 - self.sum_x.square().sum() / self.n
        return float(1.0 - self.sum_err / total.clamp(min=1e-12))


@dataclass
class SyntheticDataEvalResult:
    true_l0: float  # mean active ground-truth features per sample
    sae_l0: float  # mean active SAE latents per sample
    dead_latents: int
    shrinkage: float
    explained_variance: float
    mcc: float
    uniqueness: float
    classification: ClassificationMetrics

    def to_log_dict(self, prefix: str = "") -> dict[str, float | int]:
        d: dict[str, float | int] = {f"{prefix}{k}": v for k, v in asdict(self).items() if k != "classification"}
        d.update({f"{prefix}classification/{k}": v for k, v in asdict(self.classification).items()})
        return d

    def to_dict(self) -> dict[str, Any]:
        return asdict(self)


@torch.no_grad()
def eval_sae_on_synthetic_data(sae: Any, feature_dict: Any, activations_generator: Any, num_samples: int = 100_000,
                               batch_size: int | None = None,
                               activation_scaler: Any = None) -> SyntheticDataEvalResult:
    """Stream `num_samples` synthetic rows through the SAE and collect every metric above
    (sae_lens/synthetic/evals.py:413-502).  With `activation_scaler` the hidden activations are
    scaled before encoding and the reconstruction unscaled before it is compared with them;
    `batch_size=None` evaluates all samples in one batch."""
    if batch_size is None:
        batch_size = num_samples
    dev = next(iter(sae.parameters())).device
    W_dec = sae.W_dec.detach().float()
    gt = feature_dict.feature_vectors.detach().float()
    true_l0, l0, dead = L0Calculator(), L0Calculator(), DeadLatentsCalculator(W_dec.shape[0])
    shrink, ev = ShrinkageCalculator(), ExplainedVarianceCalculator(gt.shape[1], dev)
    cls = ClassificationMetricsCalculator(W_dec, gt)
    done = 0
    while done < num_samples:
        n = min(batch_size, num_samples - done)
        f = activations_generator.sample(n)
        true_l0.add_batch(f)
        h = feature_dict(f).to(dev)
        hs = activation_scaler.scale(h) if activation_scaler is not None else h
        lat = sae.encode(hs.to(sae.W_enc.dtype))
        out = sae.decode(lat).float()
        if activation_scaler is not None:
            out = activation_scaler.unscale(out)
        l0.add_batch(lat)
        dead.add_batch(lat)
        shrink.add_batch(out, h)
        ev.add_batch(out, h)
        cls.add_batch(lat.to(f.device) if not f.is_sparse else lat.cpu(), f if not f.is_sparse else f.cpu())
        done += n
    return SyntheticDataEvalResult(true_l0=true_l0.compute(), sae_l0=l0.compute(), dead_latents=dead.compute(),
                                   shrinkage=shrink.compute(),
                                   explained_variance=ev.compute(), mcc=mean_correlation_coefficient(W_dec, gt),
                                   uniqueness=feature_uniqueness(W_dec, gt), classification=cls.compute())
