"""Train one SAE per hook from a single LM pass (role of sae_lens/training/multi_sae_trainer.py).

The data provider yields `{hook_name: activations}` batches.  Every hook's SAE steps on its own
rows; the firing statistics are kept per hook.  Backward modes:
* "combined": sum every hook's loss and run one backward (one optimizer over all parameters);
* "sequential": one backward per hook in `forward` / `reverse` / `largest_first` order, which
  bounds peak memory to one SAE's activations.
Statistics sync across data-parallel ranks ("immediate" every step, "deferred" until the next
window boundary, "periodic" every `stats_sync_interval` steps) uses batched MAX / SUM all-reduces.
On CUDA, TopK SAEs step on their own fused native engines (each is independent).
Checkpoints hold one sub-directory per hook (weights gathered over SAE tensor parallelism, written
by the first rank of the first replica), `multi_sae_manifest.json` and the trainer state, whose
optimizer state is keyed by hook and parameter name (gathered over TP when saved, sliced when
loaded).  Resuming loads every hook's weights; under TP only the group's first rank reads the file
and scatters the shards (sae_lens/training/multi_sae_trainer.py:786-1034, 1202-1275).
"""

from __future__ import annotations

import json
import re
import time
from pathlib import Path
from typing import Any

import torch
import torch.distributed as dist
from safetensors import safe_open
from safetensors.torch import load_file, save_file

from saelens_b200.constants import (
    MULTI_SAE_MANIFEST_FILENAME,
    SAE_CFG_FILENAME,
    SAE_WEIGHTS_FILENAME,
    SPARSITY_FILENAME,
    TRAINER_STATE_FILENAME,
)
from saelens_b200.models.sae import TrainCoefficientConfig, TrainStepInput, TrainStepOutput
from saelens_b200.training.optim import CoefficientScheduler, get_lr_scheduler


def sanitize_hook_name_for_path(hook_name: str) -> str:
    return re.sub(r"[^A-Za-z0-9_.-]", "_", hook_name)


def _tp_group_of(sae: Any) -> dist.ProcessGroup | None:
    g = getattr(sae, "_tp_group", None)
    return g if (g is not None and dist.is_initialized() and dist.get_world_size(g) > 1) else None


_DTYPE_CODES = [torch.float32, torch.bfloat16, torch.float16, torch.float64, torch.int32, torch.int64,
                torch.int16, torch.int8, torch.uint8, torch.bool]


def load_tp_sharded_state_dict(filepath: str | Path, base_sae: Any, tp_group: dist.ProcessGroup) -> dict[str, torch.Tensor]:
    """This rank's shard of a full SAE checkpoint, with only the TP group's first rank reading the
    tensors: it sends every rank its slice of the sharded tensors (`_tp_param_shard_dims`) and
    broadcasts the replicated ones; the others read only the file's header (names and shapes).
    The result is already sharded: do not pass it through `process_state_dict_for_loading`."""
    rank, size = dist.get_rank(tp_group), dist.get_world_size(tp_group)
    root = dist.get_global_rank(tp_group, 0)
    dims = base_sae._tp_param_shard_dims()
    dev = base_sae.W_dec.device if dist.get_backend(tp_group) == "nccl" else torch.device("cpu")
    with safe_open(str(filepath), framework="pt", device="cpu") as f:
        names = sorted(f.keys())  # the same order on every rank
        shapes = {k: list(f.get_slice(k).get_shape()) for k in names}
    full = load_file(str(filepath)) if rank == 0 else {}
    out: dict[str, torch.Tensor] = {}
    for k in names:
        dim = dims.get(k)
        # the other ranks learn the tensor's dtype from a one-element broadcast of its code
        code = torch.tensor([_DTYPE_CODES.index(full[k].dtype) if rank == 0 else -1], device=dev)
        dist.broadcast(code, src=root, group=tp_group)
        dtype = _DTYPE_CODES[int(code.item())]
        if dim is None:
            t = full[k].to(dev) if rank == 0 else torch.empty(shapes[k], dtype=dtype, device=dev)
            dist.broadcast(t, src=root, group=tp_group)
            out[k] = t
            continue
        if shapes[k][dim] % size:
            raise ValueError(f"checkpoint tensor {k!r} has {shapes[k][dim]} entries on dim {dim}, "
                             f"not divisible by the TP size {size}")
        n = shapes[k][dim] // size
        shard_shape = list(shapes[k])
        shard_shape[dim] = n
        recv = torch.empty(shard_shape, dtype=dtype, device=dev)
        parts = [c.contiguous().to(dev) for c in full[k].split(n, dim=dim)] if rank == 0 else None
        dist.scatter(recv, parts, src=root, group=tp_group)
        out[k] = recv
    return out


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
        # full-width statistics (the TP forward returns feature activations over the whole dictionary)
        self.act_freq_scores = {h: torch.zeros(self.base_sae_by_hook[h].cfg.d_sae, device=dev) for h in self.hook_names}
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
        self.checkpoint_thresholds: list[int] = []
        n_ck = int(getattr(cfg, "n_checkpoints", 0) or 0)
        if n_ck > 0 and getattr(cfg, "checkpoint_path", None) is not None:
            every = cfg.total_training_samples / (n_ck + 1)
            self.checkpoint_thresholds = [int(every * i) for i in range(1, n_ck + 1)]

    # ---------------------------------------------------------------- helpers
    def _tp_rank(self) -> int:
        g = _tp_group_of(self.base_sae_by_hook[self.hook_names[0]])
        return dist.get_rank(g) if g is not None else 0

    def _dp_rank(self) -> int:
        return dist.get_rank(self.dp_group) if self.dp_group is not None else 0

    def _is_writer(self) -> bool:
        return self._tp_rank() == 0 and self._dp_rank() == 0

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
                base = self.base_sae_by_hook[h]
                if hasattr(base, "sync_tensor_parallel_gradients"):
                    base.sync_tensor_parallel_gradients()
                base.clip_grad_norm_(1.0)
                losses[h] = out.loss.detach()
            self.optimizer.step()
            self.optimizer.zero_grad()
            if self.lr_scheduler is not None:
                self.lr_scheduler.step()
        for d in self.coefficient_schedulers.values():
            for s in d.values():
                s.step()
        return {h: float(v) for h, v in losses.items()}

    def fit(self, quiesce_request_path: str | Path | None = None,
            quiesce_ack_path: str | Path | None = None) -> dict[str, Any]:
        """Train until the sample budget or the data ends.  With `quiesce_request_path` (a
        topology supervisor's request file) every step checks for it; on a request all ranks write
        a `quiesce_*` checkpoint, the writer acknowledges, and the run stops without a final
        checkpoint (`self.quiesced`)."""
        from saelens_b200.training.sae_trainer import agree_any

        self.quiesced = False
        first = self.base_sae_by_hook[self.hook_names[0]]
        groups = [g for g in (_tp_group_of(first), self.dp_group) if g is not None]

        def quiesce_if_requested() -> bool:
            if quiesce_request_path is None:
                return False
            if not agree_any(Path(quiesce_request_path).exists(), groups, first.W_dec.device):
                return False
            self.save_checkpoint(checkpoint_name=f"quiesce_{self.n_training_samples}")
            if quiesce_ack_path is not None and self._is_writer():
                Path(quiesce_ack_path).touch()
            self.quiesced = True
            return True

        while self.n_training_samples < self.cfg.total_training_samples:
            try:
                batch = next(self.data_provider)
            except StopIteration:
                quiesce_if_requested()  # the data can end because the producers quiesced first
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
            if self.checkpoint_thresholds and self.n_training_samples > self.checkpoint_thresholds[0]:
                self.save_checkpoint(checkpoint_name=str(self.n_training_samples))
                self.checkpoint_thresholds.pop(0)
            if quiesce_if_requested():
                return self.base_sae_by_hook
        if getattr(self.cfg, "save_final_checkpoint", False) and not self.quiesced:
            self.save_checkpoint(checkpoint_name=f"final_{self.n_training_samples}")
        return self.base_sae_by_hook

    # ---------------------------------------------------------------- checkpoints
    def _manifest(self) -> dict[str, Any]:
        return {"hook_names": self.hook_names,
                "subdirs": {h: sanitize_hook_name_for_path(h) for h in self.hook_names},
                "n_training_steps": self.n_training_steps, "n_training_samples": self.n_training_samples}

    def save_final(self, output_path: str | Path) -> None:
        """The inference SAEs, one sub-directory per hook, plus the manifest.  Every rank of the
        first data-parallel replica calls it (the TP gathers are collective); the first writes."""
        if self._dp_rank() != 0:
            return
        base = Path(output_path)
        writer = self._is_writer()
        sparsity = self.log_feature_sparsity_by_hook()
        for h in self.hook_names:
            sae = self.base_sae_by_hook[h]
            sd = {k: v.detach().contiguous() for k, v in sae.state_dict().items()}
            sae.process_state_dict_for_saving_inference(sd)  # gathers the TP shards (collective)
            if writer:
                d = base / sanitize_hook_name_for_path(h)
                d.mkdir(parents=True, exist_ok=True)
                save_file({k: v.contiguous() for k, v in sd.items()}, d / SAE_WEIGHTS_FILENAME)
                (d / SAE_CFG_FILENAME).write_text(json.dumps(sae.cfg.get_inference_sae_cfg_dict()))
                save_file({"sparsity": sparsity[h]}, d / SPARSITY_FILENAME)
        if writer:
            (base / MULTI_SAE_MANIFEST_FILENAME).write_text(json.dumps(self._manifest(), indent=2))

    def save_checkpoint(self, checkpoint_path: str | Path | None = None, checkpoint_name: str | None = None,
                        ) -> Path | None:
        """Write a checkpoint to `checkpoint_path`, or to `cfg.checkpoint_path / checkpoint_name`
        (nothing when the config has no checkpoint path).  Every rank of the first data-parallel
        replica takes part (the TP gathers are collective); the first of them writes."""
        if checkpoint_path is None:
            if checkpoint_name is None or getattr(self.cfg, "checkpoint_path", None) is None:
                return None
            checkpoint_path = Path(self.cfg.checkpoint_path) / checkpoint_name
        base = Path(checkpoint_path)
        if self._dp_rank() != 0:
            return base
        writer = self._is_writer()
        if writer:
            base.mkdir(parents=True, exist_ok=True)
        sparsity = self.log_feature_sparsity_by_hook()
        for h in self.hook_names:
            sae = self.base_sae_by_hook[h]
            sd = {k: v.detach().contiguous() for k, v in sae.state_dict().items()}
            sae.process_state_dict_for_saving(sd)  # gathers the TP shards (collective)
            if writer:
                d = base / sanitize_hook_name_for_path(h)
                d.mkdir(parents=True, exist_ok=True)
                save_file({k: v.contiguous() for k, v in sd.items()}, d / SAE_WEIGHTS_FILENAME)
                (d / SAE_CFG_FILENAME).write_text(json.dumps(sae.cfg.to_dict()))
                save_file({"sparsity": sparsity[h]}, d / SPARSITY_FILENAME)
        optim = self._named_optimizer_state()  # gathered over TP (collective)
        if writer:
            state: dict[str, Any] = {
                "format": "multi_sae_named_v2",
                "hook_names": self.hook_names,
                "n_training_steps": self.n_training_steps, "n_training_samples": self.n_training_samples,
                "act_freq_scores": self.act_freq_scores,
                "n_forward_passes_since_fired": self.n_forward_passes_since_fired,
                "n_frac_active_samples": self.n_frac_active_samples,
                "optimizer_by_hook": optim,
                "lr_scheduler": self.lr_scheduler.state_dict() if self.lr_scheduler is not None else None,
                "engines": {h: e.optimizer_state() for h, e in self.engines.items()},
                "engine_steps": {h: e.step_count for h, e in self.engines.items()},
            }
            torch.save(state, base / TRAINER_STATE_FILENAME)
            (base / MULTI_SAE_MANIFEST_FILENAME).write_text(json.dumps(self._manifest(), indent=2))
            if self.save_checkpoint_fn is not None:
                self.save_checkpoint_fn(checkpoint_path=base)
        return base

    def _named_optimizer_state(self) -> dict[str, dict[str, dict[str, Any]]]:
        """{hook: {parameter name: Adam state}} of the torch optimizer, with the TP-sharded
        parameters' moments gathered to full size."""
        out: dict[str, dict[str, dict[str, Any]]] = {}
        if self.optimizer is None:
            return out
        for h in self.hook_names:
            if h in self.engines:
                continue
            sae = self.base_sae_by_hook[h]
            st = {name: {k: (v.detach().clone() if torch.is_tensor(v) else v)
                         for k, v in self.optimizer.state.get(p, {}).items()}
                  for name, p in sae.named_parameters() if self.optimizer.state.get(p)}
            if hasattr(sae, "process_named_optimizer_state_for_saving"):
                sae.process_named_optimizer_state_for_saving(st)
            out[h] = st
        return out

    def _load_named_optimizer_state(self, by_hook: dict[str, dict[str, dict[str, Any]]]) -> None:
        assert self.optimizer is not None
        for h, st in by_hook.items():
            if h not in self.base_sae_by_hook or h in self.engines:
                continue
            sae = self.base_sae_by_hook[h]
            st = {n: dict(v) for n, v in st.items()}
            if hasattr(sae, "process_named_optimizer_state_for_loading"):
                sae.process_named_optimizer_state_for_loading(st)  # this rank's TP slice
            params = dict(sae.named_parameters())
            for name, pst in st.items():
                if name not in params:
                    continue
                p = params[name]
                self.optimizer.state[p] = {
                    k: (v.to(device=p.device, dtype=p.dtype if (v.is_floating_point() and v.ndim > 0) else v.dtype)
                        if torch.is_tensor(v) else v)
                    for k, v in pst.items()}

    def load_checkpoint_models(self, checkpoint_path: str | Path) -> None:
        """Load every hook's SAE weights from a checkpoint (one sub-directory per hook).  Under SAE
        tensor parallelism the TP group's first rank reads each file and scatters the shards."""
        for h in self.hook_names:
            f = Path(checkpoint_path) / sanitize_hook_name_for_path(h) / SAE_WEIGHTS_FILENAME
            base = self.base_sae_by_hook[h]
            g = _tp_group_of(base)
            if g is not None:
                sd = load_tp_sharded_state_dict(f, base, g)
            else:
                sd = load_file(str(f))
                base.process_state_dict_for_loading(sd)
            wrapped = self.sae_by_hook[h]
            if type(wrapped).__name__ == "FullyShardedDataParallel":
                from torch.distributed.fsdp import FullyShardedDataParallel as FSDP
                from torch.distributed.fsdp import StateDictType

                with FSDP.state_dict_type(wrapped, StateDictType.FULL_STATE_DICT):
                    wrapped.load_state_dict(sd)
            else:
                base.load_state_dict({k: v.to(base.W_dec.device) for k, v in sd.items()})
            if h in self.engines:
                self.engines[h].refresh()

    def load_trainer_state(self, checkpoint_path: str | Path) -> None:
        """Restore counters, statistics and optimizer state; the checkpoint must hold the same
        hooks (multi_sae_trainer.py resume in the reference raises on a mismatch too)."""
        man = Path(checkpoint_path) / MULTI_SAE_MANIFEST_FILENAME
        if man.exists():
            saved = json.loads(man.read_text()).get("hook_names")
            if saved is not None and list(saved) != list(self.hook_names):
                raise ValueError(f"checkpoint hooks {saved} do not match this trainer's hooks {self.hook_names}")
        if (Path(checkpoint_path) / sanitize_hook_name_for_path(self.hook_names[0]) / SAE_WEIGHTS_FILENAME).exists():
            self.load_checkpoint_models(checkpoint_path)
        st = torch.load(Path(checkpoint_path) / TRAINER_STATE_FILENAME, map_location="cpu", weights_only=False)
        self.n_training_steps = st["n_training_steps"]
        self.n_training_samples = st["n_training_samples"]
        self.act_freq_scores = {h: v.to(self.cfg.device) for h, v in st["act_freq_scores"].items()}
        self.n_forward_passes_since_fired = {h: v.to(self.cfg.device) for h, v in st["n_forward_passes_since_fired"].items()}
        self.n_frac_active_samples = st["n_frac_active_samples"]
        if self.optimizer is not None and st.get("optimizer_by_hook") is not None:
            self._load_named_optimizer_state(st["optimizer_by_hook"])
        elif self.optimizer is not None and st.get("optimizer") is not None:
            self.optimizer.load_state_dict(st["optimizer"])
        if self.lr_scheduler is not None and st.get("lr_scheduler") is not None:
            self.lr_scheduler.load_state_dict(st["lr_scheduler"])
        for h, s in st.get("engines", {}).items():
            if h in self.engines:
                self.engines[h].load_optimizer_state(s)
