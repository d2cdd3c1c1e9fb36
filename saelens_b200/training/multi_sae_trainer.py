"""Train one SAE per hook from a single LM pass (role of sae_lens/training/multi_sae_trainer.py).

The data provider yields `{hook_name: activations}` batches.  Every hook's SAE steps on its own
rows; the firing statistics are kept per hook.  Backward modes:
* "combined": sum every hook's loss and run one backward (one optimizer over all parameters);
* "sequential": one backward per hook in `forward` / `reverse` / `largest_first` order, which
  bounds peak memory to one SAE's activations.
Statistics sync across data-parallel ranks ("immediate" every step, "deferred" until the next
window boundary, "periodic" every `stats_sync_interval` steps) uses batched MAX / SUM all-reduces.
On CUDA, TopK SAEs step on their own fused native engines (each is independent).
Checkpoints hold one sub-directory per hook plus `multi_sae_manifest.json`.
"""

from __future__ import annotations

import json
import re
import time
from pathlib import Path
from typing import Any

import torch
import torch.distributed as dist
from safetensors.torch import save_file

from saelens_b200.constants import MULTI_SAE_MANIFEST_FILENAME, SPARSITY_FILENAME, TRAINER_STATE_FILENAME
from saelens_b200.models.sae import TrainCoefficientConfig, TrainStepInput, TrainStepOutput
from saelens_b200.training.optim import CoefficientScheduler, get_lr_scheduler


def sanitize_hook_name_for_path(hook_name: str) -> str:
    return re.sub(r"[^A-Za-z0-9_.-]", "_", hook_name)


class MultiSAETrainer:
    def __init__(self, *, hook_names: list[str], sae_by_hook: dict[str, Any], data_provider: Any, cfg: Any,
                 base_sae_by_hook: dict[str, Any] | None = None, save_checkpoint_fn: Any = None,
                 dp_group: dist.ProcessGroup | None = None, token_count_weighted_dp: bool = False,
                 sae_dp_mode: str = "ddp", backward_mode: str = "combined", seed_mode: str = "same") -> None:
        if backward_mode not in ("combined", "sequential"):
            raise ValueError("backward_mode must be 'combined' or 'sequential'")
        self.hook_names = list(hook_names)
        self.sae_by_hook = sae_by_hook
        self.base_sae_by_hook = base_sae_by_hook or sae_by_hook
        self.data_provider = data_provider
        self.cfg = cfg
        self.save_checkpoint_fn = save_checkpoint_fn
        self.dp_group = dp_group
        self.token_count_weighted_dp = token_count_weighted_dp
        self.sae_dp_mode = sae_dp_mode
        self.backward_mode = backward_mode
        self.seed_mode = seed_mode
        self.backward_order = getattr(cfg, "multi_sae_backward_order", "forward")
        self.stats_sync_mode = getattr(cfg, "multi_sae_stats_sync_mode", "immediate")
        self.stats_sync_interval = int(getattr(cfg, "multi_sae_stats_sync_interval", 1))
        if self.backward_order not in ("forward", "reverse", "largest_first"):
            raise ValueError("multi_sae_backward_order must be 'forward', 'reverse', or 'largest_first'")
        if self.stats_sync_mode not in ("immediate", "deferred", "periodic"):
            raise ValueError("multi_sae_stats_sync_mode must be 'immediate', 'deferred', or 'periodic'")
        if self.stats_sync_interval < 1:
            raise ValueError("multi_sae_stats_sync_interval must be >= 1")
        self.n_training_steps = 0
        self.n_training_samples = 0
        self._t0 = time.time()
        dev = cfg.device
        self.act_freq_scores = {h: torch.zeros(self.base_sae_by_hook[h].W_dec.shape[0], device=dev) for h in self.hook_names}
        self.n_forward_passes_since_fired = {h: torch.zeros_like(self.act_freq_scores[h]) for h in self.hook_names}
        self._pending_fire = {h: torch.zeros_like(self.act_freq_scores[h], dtype=torch.int32) for h in self.hook_names}
        self._pending_freq = {h: torch.zeros_like(self.act_freq_scores[h]) for h in self.hook_names}
        self.n_frac_active_samples = 0
        # native engines for TopK SAEs on CUDA (each independent); a shared Adam for the rest
        self.engines: dict[str, Any] = {}
        if getattr(cfg, "sae_engine", "auto") != "torch" and dp_group is None:
            from saelens_b200.training.engine import FusedTopKEngine, engine_supported

            for h in self.hook_names:
                if engine_supported(self.base_sae_by_hook[h]):
                    self.engines[h] = FusedTopKEngine(self.base_sae_by_hook[h], lr=cfg.lr, beta1=cfg.adam_beta1,
                                                      beta2=cfg.adam_beta2)
        params = [p for h in self.hook_names if h not in self.engines for p in self.sae_by_hook[h].parameters()]
        self.optimizer = torch.optim.Adam(params, lr=cfg.lr, betas=(cfg.adam_beta1, cfg.adam_beta2)) if params else None
        self.lr_scheduler = get_lr_scheduler(cfg.lr_scheduler_name, self.optimizer, cfg.total_training_steps, cfg.lr,
                                             cfg.lr_warm_up_steps, cfg.lr_decay_steps, cfg.lr_end, cfg.n_restart_cycles) \
            if self.optimizer is not None else None
        from saelens_b200.training.optim import LRSchedule

        self._lr_fn = LRSchedule(cfg.lr_scheduler_name, cfg.total_training_steps, cfg.lr, cfg.lr_warm_up_steps,
                                 cfg.lr_decay_steps, cfg.lr_end, cfg.n_restart_cycles)
        self.coefficient_schedulers: dict[str, dict[str, CoefficientScheduler]] = {}
        for h in self.hook_names:
            d = {}
            for name, cc in self.base_sae_by_hook[h].get_coefficients().items():
                if not isinstance(cc, TrainCoefficientConfig):
                    cc = TrainCoefficientConfig(cc, 0)
                d[name] = CoefficientScheduler(cc.warm_up_steps, cc.value)
            self.coefficient_schedulers[h] = d

    # ---------------------------------------------------------------- helpers
    def dead_neurons(self, hook: str) -> torch.Tensor:
        return self.n_forward_passes_since_fired[hook] > self.cfg.dead_feature_window

    def feature_sparsity(self, hook: str) -> torch.Tensor:
        return self.act_freq_scores[hook] / max(self.n_frac_active_samples, 1)

    def log_feature_sparsity_by_hook(self) -> dict[str, torch.Tensor]:
        return {h: torch.log10(self.feature_sparsity(h) + 1e-10).cpu() for h in self.hook_names}

    def _ordered_for_backward(self) -> list[str]:
        if self.backward_order == "reverse":
            return list(reversed(self.hook_names))
        if self.backward_order == "largest_first":
            return sorted(self.hook_names, key=lambda h: -sum(p.numel() for p in self.sae_by_hook[h].parameters()))
        return list(self.hook_names)

    def _should_sync(self) -> bool:
        if self.dp_group is None:
            return False
        if self.stats_sync_mode == "immediate":
            return True
        if self.stats_sync_mode == "periodic":
            return (self.n_training_steps + 1) % self.stats_sync_interval == 0
        return (self.n_training_steps + 1) % self.cfg.feature_sampling_window == 0

    @torch.no_grad()
    def _update_stats(self, hook: str, fired_rows: torch.Tensor) -> None:
        """`fired_rows`: per-latent number of rows in which the latent fired this step."""
        self._pending_fire[hook] = torch.maximum(self._pending_fire[hook], (fired_rows > 0).to(torch.int32))
        self._pending_freq[hook] += fired_rows.float()
        if self.dp_group is None or self._should_sync():
            if self.dp_group is not None:
                flat_fire = torch.cat([self._pending_fire[h] for h in self.hook_names])
                dist.all_reduce(flat_fire, op=dist.ReduceOp.MAX, group=self.dp_group)
                flat_freq = torch.cat([self._pending_freq[h] for h in self.hook_names])
                dist.all_reduce(flat_freq, op=dist.ReduceOp.SUM, group=self.dp_group)
                off = 0
                for h in self.hook_names:
                    n = self._pending_fire[h].numel()
                    self._pending_fire[h] = flat_fire[off : off + n]
                    self._pending_freq[h] = flat_freq[off : off + n]
                    off += n
            for h in self.hook_names:
                fired = self._pending_fire[h].bool()
                self.n_forward_passes_since_fired[h] += 1
                self.n_forward_passes_since_fired[h][fired] = 0
                self.act_freq_scores[h] += self._pending_freq[h]
                self._pending_fire[h].zero_()
                self._pending_freq[h].zero_()

    def _forward_one(self, hook: str, acts: torch.Tensor) -> TrainStepOutput:
        coeffs = {n: s.value for n, s in self.coefficient_schedulers[hook].items()}
        return self.sae_by_hook[hook](TrainStepInput(sae_in=acts, coefficients=coeffs,
                                                     dead_neuron_mask=self.dead_neurons(hook),
                                                     n_training_steps=self.n_training_steps))

    # ---------------------------------------------------------------- step
    def _train_step(self, batch: dict[str, torch.Tensor]) -> dict[str, float]:
        losses: dict[str, float] = {}
        torch_hooks = [h for h in self.hook_names if h not in self.engines]
        for h, eng in self.engines.items():
            acts = batch[h].to(eng.device)
            run_aux = self.n_training_steps >= self.cfg.dead_feature_window and bool(self.dead_neurons(h).any())
            r = eng.step(acts, lr=self._lr_fn.lr_at(self.n_training_steps), dead_mask=self.dead_neurons(h),
                         run_aux=run_aux)
            self._update_stats(h, r.fire_counts.clone())
            losses[h] = r.loss
        if torch_hooks:
            assert self.optimizer is not None
            outs: dict[str, TrainStepOutput] = {}
            if self.backward_mode == "combined":
                total = None
                for h in torch_hooks:
                    out = self._forward_one(h, batch[h])
                    outs[h] = out
                    total = out.loss if total is None else total + out.loss
                assert total is not None
                total.backward()
            else:
                for h in [x for x in self._ordered_for_backward() if x in torch_hooks]:
                    out = self._forward_one(h, batch[h])
                    out.loss.backward()
                    outs[h] = out
            for h, out in outs.items():
                with torch.no_grad():
                    fa = out.feature_acts
                    self._update_stats(h, (fa > 0).sum(0).to(torch.int32) if not fa.is_sparse else
                                       (fa.to_dense() > 0).sum(0).to(torch.int32))
                self.base_sae_by_hook[h].clip_grad_norm_(1.0)
                losses[h] = out.loss.detach()
            self.optimizer.step()
            self.optimizer.zero_grad()
            if self.lr_scheduler is not None:
                self.lr_scheduler.step()
        for d in self.coefficient_schedulers.values():
            for s in d.values():
                s.step()
        return {h: float(v) for h, v in losses.items()}

    def fit(self) -> dict[str, Any]:
        while self.n_training_samples < self.cfg.total_training_samples:
            try:
                batch = next(self.data_provider)
            except StopIteration:
                break
            if (self.n_training_steps + 1) % self.cfg.feature_sampling_window == 0:
                for h in self.hook_names:
                    self.act_freq_scores[h].zero_()
                self.n_frac_active_samples = 0
            n = next(iter(batch.values())).shape[0]
            self.n_training_samples += n
            self.n_frac_active_samples += n
            self._train_step(batch)
            self.n_training_steps += 1
        return self.base_sae_by_hook

    # ---------------------------------------------------------------- checkpoints
    def _manifest(self) -> dict[str, Any]:
        return {"hook_names": self.hook_names,
                "subdirs": {h: sanitize_hook_name_for_path(h) for h in self.hook_names},
                "n_training_steps": self.n_training_steps, "n_training_samples": self.n_training_samples}

    def save_final(self, output_path: str | Path) -> None:
        base = Path(output_path)
        base.mkdir(parents=True, exist_ok=True)
        for h in self.hook_names:
            d = base / sanitize_hook_name_for_path(h)
            self.base_sae_by_hook[h].save_inference_model(d)
            save_file({"sparsity": self.log_feature_sparsity_by_hook()[h]}, d / SPARSITY_FILENAME)
        (base / MULTI_SAE_MANIFEST_FILENAME).write_text(json.dumps(self._manifest(), indent=2))

    def save_checkpoint(self, checkpoint_path: str | Path) -> None:
        base = Path(checkpoint_path)
        base.mkdir(parents=True, exist_ok=True)
        for h in self.hook_names:
            self.base_sae_by_hook[h].save_model(base / sanitize_hook_name_for_path(h))
        state: dict[str, Any] = {
            "n_training_steps": self.n_training_steps, "n_training_samples": self.n_training_samples,
            "act_freq_scores": self.act_freq_scores, "n_forward_passes_since_fired": self.n_forward_passes_since_fired,
            "n_frac_active_samples": self.n_frac_active_samples,
            "optimizer": self.optimizer.state_dict() if self.optimizer is not None else None,
            "engines": {h: e.optimizer_state() for h, e in self.engines.items()},
            "engine_steps": {h: e.step_count for h, e in self.engines.items()},
        }
        torch.save(state, base / TRAINER_STATE_FILENAME)
        (base / MULTI_SAE_MANIFEST_FILENAME).write_text(json.dumps(self._manifest(), indent=2))

    def load_trainer_state(self, checkpoint_path: str | Path) -> None:
        """Restore counters, statistics and optimizer state; the checkpoint must hold the same
        hooks (multi_sae_trainer.py resume in the reference raises on a mismatch too)."""
        man = Path(checkpoint_path) / MULTI_SAE_MANIFEST_FILENAME
        if man.exists():
            saved = json.loads(man.read_text()).get("hook_names")
            if saved is not None and list(saved) != list(self.hook_names):
                raise ValueError(f"checkpoint hooks {saved} do not match this trainer's hooks {self.hook_names}")
        st = torch.load(Path(checkpoint_path) / TRAINER_STATE_FILENAME, map_location="cpu", weights_only=False)
        self.n_training_steps = st["n_training_steps"]
        self.n_training_samples = st["n_training_samples"]
        self.act_freq_scores = {h: v.to(self.cfg.device) for h, v in st["act_freq_scores"].items()}
        self.n_forward_passes_since_fired = {h: v.to(self.cfg.device) for h, v in st["n_forward_passes_since_fired"].items()}
        self.n_frac_active_samples = st["n_frac_active_samples"]
        if self.optimizer is not None and st.get("optimizer") is not None:
            self.optimizer.load_state_dict(st["optimizer"])
        for h, s in st.get("engines", {}).items():
            if h in self.engines:
                self.engines[h].load_optimizer_state(s)
