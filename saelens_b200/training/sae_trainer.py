"""SAE training loop (semantics of sae_lens/training/sae_trainer.py).

Per step: next batch -> activation scaler -> train step -> firing statistics, loss / timing /
memory records, checkpoints, quiesce-file check.  The train step has two implementations:

* native (TopK SAEs on CUDA): `FusedTopKEngine.step` - the whole forward, backward, clip and
  Adam as sm_100a kernels, firing statistics updated in-kernel;
* torch (every architecture, CPU or GPU): autograd + torch.optim.Adam, with manual / DDP / FSDP
  data parallelism and tensor-parallel gradient sync exactly as the reference orders them
  (sparsity all-reduce every `feature_sampling_window`, did_fire MAX all-reduce, token-count
  loss reweighting, flat gradient all-reduce, TP sync, clip at 1.0, Adam, schedulers).
"""

from __future__ import annotations

import contextlib
import json
import logging
import math
import os
import time
from collections.abc import Callable, Iterator
from copy import deepcopy
from pathlib import Path
from typing import Any, Generic, Protocol, TypeVar

import torch
import torch.distributed as dist
from safetensors.torch import save_file

from saelens_b200 import __version__
from saelens_b200.config import SAETrainerConfig
from saelens_b200.constants import (
    ACTIVATION_SCALER_CFG_FILENAME,
    FSDP_OPTIMIZER_STATE_FILENAME_TEMPLATE,
    MSE_HISTORY_FILENAME,
    SAE_CFG_FILENAME,
    SAE_WEIGHTS_FILENAME,
    SPARSITY_FILENAME,
    TIMING_HISTORY_FILENAME,
    TRAINER_STATE_FILENAME,
)
from saelens_b200.models.sae import TrainCoefficientConfig, TrainingSAE, TrainStepInput, TrainStepOutput
from saelens_b200.parallel.profiling import nccl_nvtx_range
from saelens_b200.training.activation_scaler import ActivationScaler
from saelens_b200.training.optim import CoefficientScheduler, LRSchedule, get_lr_scheduler
from saelens_b200.utils import wandb_shim as wandb
from saelens_b200.utils.misc import path_or_tmp_dir

logger = logging.getLogger(__name__)

T_TRAINING_SAE = TypeVar("T_TRAINING_SAE", bound=TrainingSAE[Any])
DataProvider = Iterator[torch.Tensor]
FSDP_OPTIMIZER_STATE_FORMAT = "fsdp_sharded"
NATIVE_FSDP_OPTIMIZER_STATE_FORMAT = "native_fsdp_latent_sharded"


class SaveCheckpointFn(Protocol):
    def __call__(self, checkpoint_path: Path | None) -> None: ...


Evaluator = Callable[[Any, DataProvider, ActivationScaler], dict[str, Any]]


def _log_feature_sparsity(feature_sparsity: torch.Tensor, eps: float = 1e-10) -> torch.Tensor:
    return torch.log10(feature_sparsity + eps).detach().cpu()


def _unwrap_item(item: Any) -> float | int:
    if callable(item):
        item = item()
    return item.item() if isinstance(item, torch.Tensor) else item


def _is_fsdp(m: Any) -> bool:
    try:
        from torch.distributed.fsdp import FullyShardedDataParallel as FSDP

        return isinstance(m, FSDP)
    except Exception:  # noqa: BLE001
        return False


def _is_ddp(m: Any) -> bool:
    from torch.nn.parallel import DistributedDataParallel as DDP

    return isinstance(m, DDP)


def agree_any(flag: bool, groups: list[Any], device: torch.device) -> bool:
    """`flag` OR-ed over every rank of `groups` (each in turn), so that ranks which check a file at
    slightly different moments still act at the same step."""
    if not groups or not (dist.is_available() and dist.is_initialized()):
        return flag
    out = bool(flag)
    for g in groups:
        dev = device if dist.get_backend(g) == "nccl" else torch.device("cpu")
        t = torch.tensor([1 if out else 0], dtype=torch.int32, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX, group=g)
        out = bool(t.item())
    return out


class SAETrainer(Generic[T_TRAINING_SAE]):
    def __init__(self, cfg: SAETrainerConfig, sae: Any, data_provider: DataProvider,
                 evaluator: Evaluator | None = None, save_checkpoint_fn: SaveCheckpointFn | None = None,
                 dp_group: dist.ProcessGroup | None = None, token_count_weighted_dp: bool = False,
                 base_sae: Any = None, append_logs: bool = False,
                 tp_input_layout: str = "replicated", native_fsdp: bool = False) -> None:
        self.sae = sae
        # "replicated": every TP rank receives the same full batch (reference semantics);
        # "row_sharded": each TP rank receives its 1/tp slice of the batch rows.
        self.tp_input_layout = tp_input_layout
        self._base_sae = base_sae if base_sae is not None else sae
        self._is_fsdp = _is_fsdp(sae)
        self._is_ddp = _is_ddp(sae)
        # sharded data parallel on the native engine (latent-sharded optimizer state, fused
        # parameter all-gather / gradient reduce-scatter); the module is not wrapped
        self._native_fsdp = bool(native_fsdp)
        self._warned_fsdp_evals = False
        self.data_provider = data_provider
        self.evaluator = evaluator
        self.activation_scaler = ActivationScaler()
        self.save_checkpoint_fn = save_checkpoint_fn
        self.cfg = cfg
        self.dp_group = dp_group
        self.token_count_weighted_dp = token_count_weighted_dp
        self.n_training_steps = 0
        self.n_training_samples = 0
        self.started_fine_tuning = False
        self._t_ready = time.time()
        self.mse_history_path: Path | None = None
        self.timing_history_path: Path | None = None
        self.memory_history_path: Path | None = None
        self.last_step_seconds = 0.0
        self._base_sae.cfg.metadata.sae_lens_training_version = str(__version__)

        if self._should_write_training_metrics():
            out = Path(cfg.output_path)  # type: ignore[arg-type]
            out.mkdir(exist_ok=True, parents=True)
            self.mse_history_path = out / MSE_HISTORY_FILENAME
            if not append_logs:
                self.mse_history_path.write_text("")
        if self._should_write_timing_metrics():
            out = Path(cfg.output_path)  # type: ignore[arg-type]
            out.mkdir(exist_ok=True, parents=True)
            self.timing_history_path = out / TIMING_HISTORY_FILENAME
            if not append_logs:
                self.timing_history_path.write_text("")
        self._memory_rank = dist.get_rank() if (dist.is_available() and dist.is_initialized()) else int(
            os.environ.get("LOCAL_RANK", "0"))
        self._profile_memory = cfg.output_path is not None and cfg.save_memory_every_n_steps > 0
        if self._profile_memory:
            out = Path(cfg.output_path)  # type: ignore[arg-type]
            out.mkdir(exist_ok=True, parents=True)
            self.memory_history_path = out / f"memory_history_rank{self._memory_rank}.jsonl"
            self.memory_history_path.write_text("")

        self.checkpoint_thresholds: list[int] = []
        if cfg.n_checkpoints > 0:
            stride = math.ceil(cfg.total_training_samples / (cfg.n_checkpoints + 1))
            self.checkpoint_thresholds = list(range(0, cfg.total_training_samples, stride))[1:]

        # firing statistics cover every latent (the PyTorch TP forward gathers the activations to
        # full width); the native TP engine keeps them per latent shard (resized below)
        d_stats = int(self._base_sae.cfg.d_sae)
        self.act_freq_scores = torch.zeros(d_stats, device=cfg.device)
        self.n_forward_passes_since_fired = torch.zeros(d_stats, device=cfg.device)
        self.n_frac_active_samples = 0

        # ---- engine selection
        self.engine: Any = None
        want = getattr(cfg, "sae_engine", "auto")
        self._engine_stats_global = False  # engine firing statistics already cover every DP rank
        if self._native_fsdp:
            from saelens_b200.parallel.fsdp_engine import FSDPTopKEngine

            fsdp_cls: Any = FSDPTopKEngine
            if type(self._base_sae).__name__ == "JumpReLUTrainingSAE":
                from saelens_b200.parallel.fsdp_jumprelu_engine import FSDPJumpReLUEngine

                fsdp_cls = FSDPJumpReLUEngine
            self.engine = fsdp_cls(self._base_sae, lr=cfg.lr, group=dp_group, beta1=cfg.adam_beta1,
                                   beta2=cfg.adam_beta2)
            self._engine_stats_global = True
        elif want != "torch" and not self._is_fsdp and (dp_group is not None or self._is_ddp):
            from saelens_b200.training.engine import engine_supported

            group = dp_group if dp_group is not None else getattr(sae, "process_group", None) or dist.group.WORLD
            tp_group = getattr(self._base_sae, "_tp_group", None)
            if engine_supported(self._base_sae) and tp_group is None:
                from saelens_b200.parallel.ddp_engine import DDPTopKEngine

                self.engine = DDPTopKEngine(self._base_sae, lr=cfg.lr, group=group, beta1=cfg.adam_beta1,
                                            beta2=cfg.adam_beta2)
                self._engine_stats_global = True
            elif engine_supported(self._base_sae) and getattr(cfg, "tp_exchange", "p2p") == "p2p":
                from saelens_b200.parallel.tp_engine import TPTopKEngine

                self.engine = TPTopKEngine(self._base_sae, lr=cfg.lr, group=tp_group, beta1=cfg.adam_beta1,
                                           beta2=cfg.adam_beta2, input_layout=tp_input_layout, fused=True,
                                           dp_group=group)
                self._engine_stats_global = True
            elif want == "native":
                raise ValueError("sae_engine='native' requested but this SAE/device is not supported by the fused engine")
        elif want != "torch" and not (self._is_ddp or self._is_fsdp) and dp_group is None:
            from saelens_b200.training.engine import FusedTopKEngine, engine_supported

            tp_group = getattr(self._base_sae, "_tp_group", None)
            if engine_supported(self._base_sae) and tp_group is not None:
                from saelens_b200.parallel.tp_engine import TPTopKEngine

                self.engine = TPTopKEngine(self._base_sae, lr=cfg.lr, group=tp_group, beta1=cfg.adam_beta1,
                                           beta2=cfg.adam_beta2, input_layout=tp_input_layout,
                                           fused=getattr(cfg, "tp_exchange", "p2p") == "p2p")
            elif tp_group is None and type(self._base_sae).__name__ == "JumpReLUTrainingSAE" and \
                    self._jumprelu_native_ok(want == "native"):
                # dense tcgen05 step while many latents are active, the sparse step once rows are sparse
                from saelens_b200.training.jumprelu_engine import JumpReLUEngine

                self.engine = JumpReLUEngine(self._base_sae, lr=cfg.lr, beta1=cfg.adam_beta1, beta2=cfg.adam_beta2)
            elif engine_supported(self._base_sae) and tp_group is None:
                self.engine = FusedTopKEngine(self._base_sae, lr=cfg.lr, beta1=cfg.adam_beta1,
                                              beta2=cfg.adam_beta2)
            elif tp_group is None and self._matryoshka_native_ok():
                from saelens_b200.training.matryoshka_engine import MatryoshkaEngine

                self.engine = MatryoshkaEngine(self._base_sae, lr=cfg.lr, beta1=cfg.adam_beta1, beta2=cfg.adam_beta2)
            elif tp_group is None and self._dense_engine_class() is not None:
                # Standard (L1) / Gated: the dense step on the tcgen05 GEMM family
                self.engine = self._dense_engine_class()(self._base_sae, lr=cfg.lr, beta1=cfg.adam_beta1,
                                                         beta2=cfg.adam_beta2)
            elif want == "native":
                raise ValueError("sae_engine='native' requested but this SAE/device is not supported by the fused engine")

        from saelens_b200.parallel.tp_engine import TPTopKEngine

        if isinstance(self.engine, TPTopKEngine):
            n_local = int(self.engine.N)
            self.act_freq_scores = torch.zeros(n_local, device=cfg.device)
            self.n_forward_passes_since_fired = torch.zeros(n_local, device=cfg.device)
        assert cfg.lr_end is not None
        if self.engine is None:
            self.optimizer: torch.optim.Optimizer | None = torch.optim.Adam(
                sae.parameters(), lr=cfg.lr, betas=(cfg.adam_beta1, cfg.adam_beta2))
            self.lr_scheduler: Any = get_lr_scheduler(
                cfg.lr_scheduler_name, lr=cfg.lr, optimizer=self.optimizer, warm_up_steps=cfg.lr_warm_up_steps,
                decay_steps=cfg.lr_decay_steps, training_steps=cfg.total_training_steps, lr_end=cfg.lr_end,
                num_cycles=cfg.n_restart_cycles)
        else:
            self.optimizer = None
            self.lr_scheduler = LRSchedule(cfg.lr_scheduler_name, cfg.total_training_steps, cfg.lr,
                                           cfg.lr_warm_up_steps, cfg.lr_decay_steps, cfg.lr_end, cfg.n_restart_cycles)
        self.coefficient_schedulers: dict[str, CoefficientScheduler] = {}
        for name, cc in self._base_sae.get_coefficients().items():
            if not isinstance(cc, TrainCoefficientConfig):
                cc = TrainCoefficientConfig(value=cc, warm_up_steps=0)
            self.coefficient_schedulers[name] = CoefficientScheduler(cc.warm_up_steps, cc.value)
        dev_type = torch.device(cfg.device).type
        self.grad_scaler = torch.amp.GradScaler(device=dev_type, enabled=cfg.autocast and dev_type == "cuda")
        self.autocast_if_enabled = (
            torch.autocast(device_type=dev_type, dtype=torch.bfloat16, enabled=cfg.autocast)
            if cfg.autocast else contextlib.nullcontext()
        )

    # ------------------------------------------------------------------ properties
    @property
    def feature_sparsity(self) -> torch.Tensor:
        return self.act_freq_scores / max(self.n_frac_active_samples, 1)

    @property
    def base_sae(self) -> Any:
        return self._base_sae

    @property
    def sae_dp_mode(self) -> str:
        return "fsdp" if (self._is_fsdp or self._native_fsdp) else ("ddp" if self._is_ddp else "manual")

    @property
    def log_feature_sparsity(self) -> torch.Tensor:
        return _log_feature_sparsity(self.feature_sparsity)

    @property
    def dead_neurons(self) -> torch.Tensor:
        return (self.n_forward_passes_since_fired > self.cfg.dead_feature_window).bool()

    def current_lr(self) -> float:
        if self.optimizer is not None:
            return float(self.optimizer.param_groups[0]["lr"])
        return float(self.lr_scheduler.lr_at(self.lr_scheduler.step_count))

    # ------------------------------------------------------------------ loop
    def fit(self, quiesce_request_path: Path | str | None = None,
            quiesce_ack_path: Path | str | None = None) -> Any:
        self._prepare_fit()

        def quiesce_if_requested() -> bool:
            if quiesce_request_path is None:
                return False
            # every rank of the trainer takes the same decision at the same step (the checkpoint
            # gathers are collective): a request seen by any rank counts for all
            if not agree_any(Path(quiesce_request_path).exists(), self._trainer_groups(), self._base_sae.W_dec.device):
                return False
            self.save_checkpoint(checkpoint_name=f"quiesce_{self.n_training_samples}")
            if quiesce_ack_path is not None and self._is_metric_writer_rank():
                Path(quiesce_ack_path).touch()
            self.quiesced = True  # the run continues after a restart: no final checkpoint
            return True

        while self.n_training_samples < self.cfg.total_training_samples:
            if not self._fit_one_step():
                # the data can end because the producers quiesced first: quiesce, do not finish
                quiesce_if_requested()
                break
            if quiesce_if_requested():
                break
        return self._finish_fit()

    def _trainer_groups(self) -> list[Any]:
        return [g for g in (getattr(self._base_sae, "_tp_group", None), self.dp_group) if g is not None]

    def _matryoshka_native_ok(self) -> bool:
        from saelens_b200.training.matryoshka_engine import matryoshka_engine_supported

        return matryoshka_engine_supported(self._base_sae)

    def _dense_engine_class(self) -> Any:
        from saelens_b200.training.dense_engine import dense_engine_class

        return dense_engine_class(self._base_sae)

    def _jumprelu_native_ok(self, required: bool) -> bool:
        from saelens_b200.training.jumprelu_engine import jumprelu_engine_supported

        ok = jumprelu_engine_supported(self._base_sae)
        if required and not ok:
            raise ValueError("sae_engine='native' requested but this JumpReLU SAE/device is not supported")
        return ok

    def fit_steps(self, n_steps: int, read_loss: bool = True) -> list[float]:
        """Run `n_steps` iterations of the training loop (same body as `fit`).

        With `read_loss` every step's loss is copied to the host (a device->host read per step),
        which is what an interactive training loop or a progress bar does.
        """
        self._prepare_fit()
        losses: list[float] = []
        for _ in range(n_steps):
            out = self._fit_one_step()
            if out is None:
                break
            if read_loss:
                losses.append(float(out.loss.detach().to("cpu", non_blocking=False)))
        return losses

    def _prepare_fit(self) -> None:
        if getattr(self, "_fit_prepared", False):
            return
        self._fit_prepared = True
        if self.engine is None:
            self.sae.to(self.cfg.device)
        if self._base_sae.cfg.normalize_activations == "expected_average_only_in":
            self.activation_scaler.estimate_scaling_factor(self._base_sae.cfg.d_in, self.data_provider, 1000)

    def _fit_one_step(self) -> TrainStepOutput | None:
        t_wall = time.perf_counter()
        self._maybe_sync()
        try:
            batch = next(self.data_provider).to(self._base_sae.W_dec.device, non_blocking=True)
        except StopIteration:
            return None
        self._maybe_sync()
        timing = self._consume_data_provider_timing()
        rows = batch.shape[0]
        if self.engine is not None and getattr(self.engine, "input_layout", "") == "row_sharded":
            rows *= self.engine.size
        self.n_training_samples += rows
        scaled = self.activation_scaler(batch)
        self._maybe_sync()
        t0 = time.perf_counter()
        out, _, mem = self._train_step(sae=self.sae, sae_in=scaled)
        self._maybe_sync()
        sae_t = time.perf_counter() - t0
        self.last_step_seconds = sae_t
        if self.cfg.logger.log_to_wandb:
            self._log_train_step(out)
            self._run_and_log_evals()
        self._record_mse_if_needed(out)
        self._record_timing_if_needed(timing["vllm_step_time_s"], timing["transfer_time_s"], sae_t,
                                      time.perf_counter() - t_wall)
        self._record_memory_if_needed(mem)
        self._checkpoint_if_needed()
        self.n_training_steps += 1
        return out

    def _finish_fit(self) -> Any:
        if getattr(self, "quiesced", False):
            return self._base_sae
        if self.activation_scaler.scaling_factor is not None:
            self._base_sae.fold_activation_norm_scaling_factor(self.activation_scaler.scaling_factor)
            if self.engine is not None:
                self.engine.refresh()
            self.activation_scaler.scaling_factor = None
        if self.cfg.save_final_checkpoint:
            self.save_checkpoint(checkpoint_name=f"final_{self.n_training_samples}")
        if self._native_fsdp:
            self.engine.restore_full_module()
        return self._base_sae

    # ------------------------------------------------------------------ one step
    def _train_step(self, sae: Any, sae_in: torch.Tensor) -> tuple[TrainStepOutput, float, dict[str, float]]:
        if self.engine is not None:
            return self._train_step_native(sae_in)
        return self._train_step_torch(sae, sae_in)

    def _sparsity_window_tick(self) -> None:
        if (self.n_training_steps + 1) % self.cfg.feature_sampling_window == 0:
            if self.dp_group is not None and not self._engine_stats_global:
                with nccl_nvtx_range("nccl:sae_dp_sparsity_all_reduce", self.dp_group):
                    dist.all_reduce(self.act_freq_scores, op=dist.ReduceOp.SUM, group=self.dp_group)
                self.n_frac_active_samples *= dist.get_world_size(self.dp_group)
            if self.cfg.logger.log_to_wandb:
                wandb.log(self._build_sparsity_log_dict(), step=self.n_training_steps)
            self._reset_running_sparsity_stats()

    def _train_step_native(self, sae_in: torch.Tensor) -> tuple[TrainStepOutput, float, dict[str, float]]:
        self._sparsity_window_tick()
        run_aux = self.n_training_steps >= self.cfg.dead_feature_window and bool(self.dead_neurons.any())
        want_out = self._is_logging_step() or self.mse_history_path is not None
        if hasattr(self.engine, "set_coefficients"):
            self.engine.set_coefficients(self.get_coefficients())
        res = self.engine.step(sae_in, lr=self.current_lr(), dead_mask=self.dead_neurons if run_aux else None,
                               want_sae_out=want_out, act_freq=self.act_freq_scores,
                               since_fired=self.n_forward_passes_since_fired, run_aux=run_aux)
        world = 1
        if self._engine_stats_global:
            dpg = getattr(self.engine, "_dp", None)
            world = dpg.size if dpg is not None else dist.get_world_size(self.engine.group)
        self.n_frac_active_samples += self.cfg.train_batch_size_samples * world
        self.lr_scheduler.step()
        for s in self.coefficient_schedulers.values():
            s.step()
        losses = {"mse_loss": res.mse_loss, getattr(self.engine, "aux_loss_name", "auxiliary_reconstruction_loss"): res.aux_loss}
        if res.extra_losses:
            losses.update(res.extra_losses)
        d_sae = self._base_sae.cfg.d_sae
        out = TrainStepOutput(
            sae_in=sae_in, sae_out=res.sae_out if res.sae_out is not None else sae_in.new_empty(0),
            feature_acts=_LazySparse(res, d_sae), hidden_pre=sae_in.new_empty(0), loss=res.loss, losses=losses,
        )
        out.metrics["grad_norm"] = self.engine.grad_norm
        return out, 0.0, {}

    def _train_step_torch(self, sae: Any, sae_in: torch.Tensor) -> tuple[TrainStepOutput, float, dict[str, float]]:
        sae.train()
        self._sparsity_window_tick()
        step_input = TrainStepInput(sae_in=sae_in, dead_neuron_mask=self.dead_neurons,
                                    coefficients=self.get_coefficients(), n_training_steps=self.n_training_steps,
                                    is_logging_step=self._is_logging_step())
        cuda = torch.cuda.is_available() and self._base_sae.W_dec.is_cuda
        if self._profile_memory and cuda:
            torch.cuda.reset_peak_memory_stats()
        with self.autocast_if_enabled:
            ctx = nccl_nvtx_range("nccl:sae_fsdp_forward_param_all_gather", self.dp_group) if self._is_fsdp \
                else contextlib.nullcontext()
            with ctx:
                out: TrainStepOutput = self.sae(step_input)
        mem: dict[str, float] = {}
        if self._profile_memory and cuda:
            mem["peak_forward_allocated_mb"] = torch.cuda.max_memory_allocated() / 2**20
            mem["peak_forward_reserved_mb"] = torch.cuda.max_memory_reserved() / 2**20
            torch.cuda.reset_peak_memory_stats()
        with torch.no_grad():
            fa = out.feature_acts
            firing = fa.bool().float()
            did_fire = firing.sum(-2).bool()
            if did_fire.is_sparse:
                did_fire = did_fire.to_dense()
            if self.dp_group is not None:
                df = did_fire.to(torch.int32)
                with nccl_nvtx_range("nccl:sae_dp_did_fire_all_reduce", self.dp_group):
                    dist.all_reduce(df, op=dist.ReduceOp.MAX, group=self.dp_group)
                did_fire = df.bool()
            self.n_forward_passes_since_fired += 1
            self.n_forward_passes_since_fired[did_fire] = 0
            fs = firing.sum(0)
            self.act_freq_scores += fs.to_dense() if fs.is_sparse else fs
            self.n_frac_active_samples += self.cfg.train_batch_size_samples
        loss = out.loss
        if self._is_ddp and self.dp_group is not None and self.token_count_weighted_dp:
            local = float(sae_in.shape[0])
            tok = torch.tensor(local, device=loss.device)
            with nccl_nvtx_range("nccl:sae_ddp_token_count_all_reduce", self.dp_group):
                dist.all_reduce(tok, op=dist.ReduceOp.SUM, group=self.dp_group)
            loss = loss * (local * dist.get_world_size(self.dp_group) / tok.item())
        bctx = nccl_nvtx_range(f"nccl:sae_{self.sae_dp_mode}_backward", self.dp_group) \
            if (self._is_fsdp or self._is_ddp) else contextlib.nullcontext()
        with bctx:
            self.grad_scaler.scale(loss).backward()
        assert self.optimizer is not None
        self.grad_scaler.unscale_(self.optimizer)
        if not (self._is_fsdp or self._is_ddp) and self.dp_group is not None:
            self._manual_dp_allreduce(sae_in.shape[0])
        self._base_sae.sync_tensor_parallel_gradients()
        self._base_sae.clip_grad_norm_(1.0, dp_group=self.dp_group if self._is_fsdp else None)
        if self._profile_memory and cuda:
            mem["peak_backward_allocated_mb"] = torch.cuda.max_memory_allocated() / 2**20
            mem["peak_backward_reserved_mb"] = torch.cuda.max_memory_reserved() / 2**20
            torch.cuda.reset_peak_memory_stats()
        self.grad_scaler.step(self.optimizer)
        self.grad_scaler.update()
        self.optimizer.zero_grad()
        self.lr_scheduler.step()
        for s in self.coefficient_schedulers.values():
            s.step()
        if self._profile_memory and cuda:
            mem["peak_optimizer_allocated_mb"] = torch.cuda.max_memory_allocated() / 2**20
            mem["peak_optimizer_reserved_mb"] = torch.cuda.max_memory_reserved() / 2**20
            mem["peak_step_allocated_mb"] = max(v for k, v in mem.items() if "allocated" in k)
            mem["peak_step_reserved_mb"] = max(v for k, v in mem.items() if "reserved" in k)
        return out, 0.0, mem

    def _manual_dp_allreduce(self, local_rows: int) -> None:
        grads = [p.grad for p in self._base_sae.parameters() if p.grad is not None]
        if not grads:
            return
        flat = torch.cat([g.reshape(-1) for g in grads])
        if self.token_count_weighted_dp:
            flat.mul_(float(local_rows))
            with nccl_nvtx_range("nccl:sae_manual_dp_grad_all_reduce", self.dp_group):
                dist.all_reduce(flat, group=self.dp_group)
            tok = torch.tensor(float(local_rows), device=flat.device)
            with nccl_nvtx_range("nccl:sae_manual_dp_token_count_all_reduce", self.dp_group):
                dist.all_reduce(tok, op=dist.ReduceOp.SUM, group=self.dp_group)
            flat.div_(tok.item())
        else:
            with nccl_nvtx_range("nccl:sae_manual_dp_grad_all_reduce", self.dp_group):
                dist.all_reduce(flat, group=self.dp_group)
            flat /= dist.get_world_size(self.dp_group)
        off = 0
        for g in grads:
            n = g.numel()
            g.copy_(flat[off : off + n].view_as(g))
            off += n

    # ------------------------------------------------------------------ checkpoints
    def save_checkpoint(self, checkpoint_name: str, wandb_aliases: list[str] | None = None) -> None:
        tp_group = getattr(self._base_sae, "_tp_group", None)
        tp_rank = dist.get_rank(tp_group) if tp_group is not None else 0
        dp_rank = dist.get_rank(self.dp_group) if self.dp_group is not None else 0
        if dp_rank != 0 and not (self._is_fsdp or self._native_fsdp):
            return
        ckpt: Path | None = None
        if self.cfg.checkpoint_path is not None or self.cfg.logger.log_to_wandb:
            with path_or_tmp_dir(self.cfg.checkpoint_path) as base:
                ckpt = base / checkpoint_name
                ckpt.mkdir(exist_ok=True, parents=True)
                wpath, cpath = self._save_model(ckpt)
                spath = ckpt / SPARSITY_FILENAME
                if dp_rank == 0 and tp_rank == 0:
                    save_file({"sparsity": self.log_feature_sparsity}, spath)
                self.save_trainer_state(ckpt)
                if self.cfg.logger.log_to_wandb and dp_rank == 0 and tp_rank == 0:
                    self.cfg.logger.log(self, wpath, cpath, sparsity_path=spath, wandb_aliases=wandb_aliases)
        if self.save_checkpoint_fn is not None and tp_rank == 0:
            self.save_checkpoint_fn(checkpoint_path=ckpt)
        if self._native_fsdp and self.dp_group is not None:
            dist.barrier(group=self.dp_group)  # every rank's shard and rank 0's files are written

    def _save_model(self, path: Path) -> tuple[Path, Path]:
        if self._native_fsdp:
            full = self.engine.full_weights()  # collective
            sd = {k: v.detach().cpu() for k, v in self._base_sae.state_dict().items()}
            sd.update({k: v.detach().cpu() for k, v in full.items()})
            self._base_sae.process_state_dict_for_saving(sd)
            wpath, cpath = path / SAE_WEIGHTS_FILENAME, path / SAE_CFG_FILENAME
            if dist.get_rank(self.dp_group) == 0:
                save_file({k: v.contiguous() for k, v in sd.items()}, wpath)
                with open(cpath, "w") as f:
                    json.dump(self._base_sae.cfg.to_dict(), f)
            return wpath, cpath
        if not self._is_fsdp:
            return self._base_sae.save_model(str(path))
        from torch.distributed.fsdp import FullStateDictConfig, StateDictType
        from torch.distributed.fsdp import FullyShardedDataParallel as FSDP

        with FSDP.state_dict_type(self.sae, StateDictType.FULL_STATE_DICT,
                                  FullStateDictConfig(offload_to_cpu=True, rank0_only=True)):
            sd = self.sae.state_dict()
        self._base_sae.process_state_dict_for_saving(sd)
        wpath, cpath = path / SAE_WEIGHTS_FILENAME, path / SAE_CFG_FILENAME
        tp_group = getattr(self._base_sae, "_tp_group", None)
        tp_rank = dist.get_rank(tp_group) if tp_group is not None else 0
        dp_rank = dist.get_rank(self.dp_group) if self.dp_group is not None else 0
        if dp_rank == 0 and tp_rank == 0:
            save_file({k: v.contiguous() for k, v in sd.items()}, wpath)
            with open(cpath, "w") as f:
                json.dump(self._base_sae.cfg.to_dict(), f)
        if tp_group is not None:
            dist.barrier(group=tp_group)
        return wpath, cpath

    def save_trainer_state(self, checkpoint_path: Path) -> None:
        checkpoint_path.mkdir(exist_ok=True, parents=True)
        sched = {n: s.state_dict() for n, s in self.coefficient_schedulers.items()}
        tp_group = getattr(self._base_sae, "_tp_group", None)
        tp_rank = dist.get_rank(tp_group) if tp_group is not None else 0
        dp_rank = dist.get_rank(self.dp_group) if self.dp_group is not None else 0
        dp_size = dist.get_world_size(self.dp_group) if self.dp_group is not None else 1
        if self._native_fsdp:
            shard = {n: {k: (v.detach().cpu() if torch.is_tensor(v) else v) for k, v in s.items()}
                     for n, s in self.engine.optimizer_state().items()}
            torch.save(shard, self._fsdp_optimizer_state_path(checkpoint_path))
            if dp_rank != 0:
                return
            opt_state: dict[str, Any] = {"optimizer_state_format": NATIVE_FSDP_OPTIMIZER_STATE_FORMAT,
                                         "fsdp_dp_size": dp_size}
        elif self._is_fsdp:
            self._save_fsdp_optimizer_state(checkpoint_path)
            if dp_rank != 0 or tp_rank != 0:
                return
            opt_state = {"optimizer_state_format": FSDP_OPTIMIZER_STATE_FORMAT, "fsdp_dp_size": dp_size}
        else:
            by_name = self._build_named_optimizer_state_for_save()
            if tp_rank != 0:
                return
            opt_state = {"optimizer_by_name": by_name}
        tp_size = dist.get_world_size(tp_group) if tp_group is not None else 1
        torch.save({
            **opt_state,
            "lr_scheduler": self.lr_scheduler.state_dict(),
            "n_training_samples": self.n_training_samples,
            "n_training_steps": self.n_training_steps,
            "act_freq_scores": self.act_freq_scores,
            "n_forward_passes_since_fired": self.n_forward_passes_since_fired,
            "n_frac_active_samples": self.n_frac_active_samples,
            "started_fine_tuning": self.started_fine_tuning,
            "coefficient_schedulers": sched,
            "sae_dp_mode": self.sae_dp_mode,
            "elapsed_s": time.time() - self._t_ready,
            "sae_tp_size": tp_size,
            "engine": "native" if self.engine is not None else "torch",
        }, str(checkpoint_path / TRAINER_STATE_FILENAME))
        self.activation_scaler.save(str(checkpoint_path / ACTIVATION_SCALER_CFG_FILENAME))

    def load_trainer_state(self, checkpoint_path: Path | str, skip_optimizer: bool = False) -> None:
        checkpoint_path = Path(checkpoint_path)
        self.activation_scaler.load(checkpoint_path / ACTIVATION_SCALER_CFG_FILENAME)
        st = torch.load(checkpoint_path / TRAINER_STATE_FILENAME, map_location="cpu", weights_only=False)
        if not skip_optimizer:
            saved = st.get("sae_dp_mode", "manual")
            if saved != self.sae_dp_mode:
                raise ValueError(
                    f"Cannot resume: checkpoint was saved with sae_dp_mode='{saved}' but current mode is "
                    f"'{self.sae_dp_mode}'. Cross-mode optimizer resume is not supported."
                )
            if self._native_fsdp:
                if st.get("optimizer_state_format") != NATIVE_FSDP_OPTIMIZER_STATE_FORMAT:
                    raise ValueError("Cannot resume: checkpoint was not written by the native sharded engine "
                                     f"(optimizer_state_format='{st.get('optimizer_state_format')}').")
                cur = dist.get_world_size(self.dp_group) if self.dp_group is not None else 1
                if st.get("fsdp_dp_size") != cur:
                    raise ValueError(
                        "Cannot resume FSDP checkpoint with a different sae_dp_size: checkpoint has "
                        f"{st.get('fsdp_dp_size')}, current run has {cur}."
                    )
                shard = torch.load(self._fsdp_optimizer_state_path(checkpoint_path), map_location="cpu",
                                   weights_only=False)
                self.engine.load_optimizer_state(shard)
            elif self._is_fsdp:
                if st.get("optimizer_state_format") != FSDP_OPTIMIZER_STATE_FORMAT:
                    raise ValueError(f"Cannot resume FSDP checkpoint: missing optimizer_state_format='{FSDP_OPTIMIZER_STATE_FORMAT}'.")
                cur = dist.get_world_size(self.dp_group) if self.dp_group is not None else 1
                if st.get("fsdp_dp_size") != cur:
                    raise ValueError(
                        "Cannot resume FSDP checkpoint with a different sae_dp_size: checkpoint has "
                        f"{st.get('fsdp_dp_size')}, current run has {cur}."
                    )
                self._load_fsdp_optimizer_state(checkpoint_path)
            elif "optimizer_by_name" in st:
                self._load_named_optimizer_state(st["optimizer_by_name"])
            elif self.optimizer is not None:
                self.optimizer.load_state_dict(st["optimizer"])
            self.lr_scheduler.load_state_dict(st["lr_scheduler"])
        self.n_training_samples = st["n_training_samples"]
        self.n_training_steps = st["n_training_steps"]
        self.act_freq_scores = st["act_freq_scores"].to(self.cfg.device)
        self.n_forward_passes_since_fired = st["n_forward_passes_since_fired"].to(self.cfg.device)
        self.n_frac_active_samples = st["n_frac_active_samples"]
        self.started_fine_tuning = st["started_fine_tuning"]
        for n, s in st["coefficient_schedulers"].items():
            self.coefficient_schedulers[n].load_state_dict(s)
        if "elapsed_s" in st:
            self._t_ready = time.time() - st["elapsed_s"]

    def _fsdp_optimizer_state_path(self, checkpoint_path: Path) -> Path:
        r = dist.get_rank(self.dp_group) if self.dp_group is not None else 0
        return checkpoint_path / FSDP_OPTIMIZER_STATE_FILENAME_TEMPLATE.format(rank=r)

    def _save_fsdp_optimizer_state(self, checkpoint_path: Path) -> None:
        from torch.distributed.fsdp import ShardedOptimStateDictConfig, ShardedStateDictConfig, StateDictType
        from torch.distributed.fsdp import FullyShardedDataParallel as FSDP

        with FSDP.state_dict_type(self.sae, StateDictType.SHARDED_STATE_DICT,
                                  ShardedStateDictConfig(offload_to_cpu=True),
                                  ShardedOptimStateDictConfig(offload_to_cpu=True)):
            st = FSDP.optim_state_dict(self.sae, self.optimizer, group=self.dp_group)
        torch.save(st, self._fsdp_optimizer_state_path(checkpoint_path))

    def _load_fsdp_optimizer_state(self, checkpoint_path: Path) -> None:
        from torch.distributed.fsdp import ShardedOptimStateDictConfig, ShardedStateDictConfig, StateDictType
        from torch.distributed.fsdp import FullyShardedDataParallel as FSDP

        st = torch.load(self._fsdp_optimizer_state_path(checkpoint_path), map_location="cpu", weights_only=False)
        with FSDP.state_dict_type(self.sae, StateDictType.SHARDED_STATE_DICT,
                                  ShardedStateDictConfig(offload_to_cpu=True),
                                  ShardedOptimStateDictConfig(offload_to_cpu=True)):
            st = FSDP.optim_state_dict_to_load(self.sae, self.optimizer, st, group=self.dp_group)
        assert self.optimizer is not None
        self.optimizer.load_state_dict(st)

    def _build_named_optimizer_state_for_save(self) -> dict[str, dict[str, Any]]:
        if self.engine is not None:
            by_name = {n: {k: (v.detach().clone() if torch.is_tensor(v) else deepcopy(v)) for k, v in s.items()}
                       for n, s in self.engine.optimizer_state().items()}
        else:
            by_name = {}
            assert self.optimizer is not None
            for name, p in self._base_sae.named_parameters():
                s = self.optimizer.state.get(p)
                if s:
                    by_name[name] = {k: (v.detach().clone() if torch.is_tensor(v) else deepcopy(v)) for k, v in s.items()}
        self._base_sae.process_named_optimizer_state_for_saving(by_name)
        return by_name

    def _load_named_optimizer_state(self, by_name: dict[str, dict[str, Any]]) -> None:
        by_name = deepcopy(by_name)
        self._base_sae.process_named_optimizer_state_for_loading(by_name)
        if self.engine is not None:
            self.engine.load_optimizer_state(by_name)
            return
        assert self.optimizer is not None
        self.optimizer.state.clear()
        params = dict(self._base_sae.named_parameters())
        for name, s in by_name.items():
            if name not in params:
                continue
            p = params[name]
            self.optimizer.state[p] = {
                k: (v.to(device=p.device, dtype=p.dtype if (v.is_floating_point() and v.ndim > 0) else v.dtype)
                    if torch.is_tensor(v) else deepcopy(v))
                for k, v in s.items()
            }

    # ------------------------------------------------------------------ logging helpers
    def _is_logging_step(self) -> bool:
        return self.cfg.logger.log_to_wandb and (self.n_training_steps + 1) % self.cfg.logger.wandb_log_frequency == 0

    def _should_write_training_metrics(self) -> bool:
        return self.cfg.output_path is not None and self.cfg.save_mse_every_n_steps > 0 and self._is_metric_writer_rank()

    def _should_write_timing_metrics(self) -> bool:
        return self.cfg.output_path is not None and self.cfg.save_timing_every_n_steps > 0 and self._is_metric_writer_rank()

    def _is_metric_writer_rank(self) -> bool:
        tp_group = getattr(self._base_sae, "_tp_group", None)
        tp_rank = dist.get_rank(tp_group) if (dist.is_available() and dist.is_initialized() and tp_group is not None) else 0
        dp_rank = dist.get_rank(self.dp_group) if self.dp_group is not None else 0
        return tp_rank == 0 and dp_rank == 0

    def _maybe_sync(self) -> None:
        if self.cfg.synchronize_timing and torch.cuda.is_available() and self._base_sae.W_dec.is_cuda:
            torch.cuda.synchronize()

    def _consume_data_provider_timing(self) -> dict[str, float]:
        fn = getattr(self.data_provider, "consume_last_data_timing", None)
        if fn is None:
            return {"vllm_step_time_s": 0.0, "transfer_time_s": 0.0}
        t = fn()
        return {"vllm_step_time_s": float(t.get("vllm_step_time_s", 0.0)),
                "transfer_time_s": float(t.get("transfer_time_s", 0.0))}

    @torch.no_grad()
    def _record_mse_if_needed(self, out: TrainStepOutput) -> None:
        if self.mse_history_path is None or (self.n_training_steps + 1) % self.cfg.save_mse_every_n_steps != 0:
            return
        mse = out.losses.get("mse_loss")
        if mse is None:
            mse = (out.sae_out - out.sae_in).pow(2).mean()
        rec = {"step": self.n_training_steps + 1, "n_training_samples": self.n_training_samples,
               "mse_loss": _unwrap_item(mse), "overall_loss": _unwrap_item(out.loss)}
        if "auxiliary_reconstruction_loss" in out.losses:
            rec["auxiliary_reconstruction_loss"] = _unwrap_item(out.losses["auxiliary_reconstruction_loss"])
        with open(self.mse_history_path, "a") as f:
            f.write(json.dumps(rec) + "\n")

    def _record_timing_if_needed(self, vllm_s: float, transfer_s: float, sae_s: float, wall_s: float = 0.0) -> None:
        if self.timing_history_path is None or (self.n_training_steps + 1) % self.cfg.save_timing_every_n_steps != 0:
            return
        data_s = vllm_s + transfer_s
        rec = {"step": self.n_training_steps + 1, "n_training_samples": self.n_training_samples,
               "elapsed_s": time.time() - self._t_ready, "wall_time_s": wall_s, "vllm_step_time_s": vllm_s,
               "transfer_time_s": transfer_s, "data_time_s": data_s, "vllm_time_s": data_s, "sae_time_s": sae_s,
               "step_time_s": data_s + sae_s}
        with open(self.timing_history_path, "a") as f:
            f.write(json.dumps(rec) + "\n")

    def _record_memory_if_needed(self, mem: dict[str, float]) -> None:
        if self.memory_history_path is None or (self.n_training_steps + 1) % self.cfg.save_memory_every_n_steps != 0:
            return
        with open(self.memory_history_path, "a") as f:
            f.write(json.dumps({"step": self.n_training_steps + 1, "n_training_samples": self.n_training_samples,
                                "rank": self._memory_rank, **mem}) + "\n")

    def _log_train_step(self, out: TrainStepOutput) -> None:
        if self._is_logging_step():
            wandb.log(self._build_train_step_log_dict(out, self.n_training_samples), step=self.n_training_steps)

    @torch.no_grad()
    def get_coefficients(self) -> dict[str, float]:
        return {n: s.value for n, s in self.coefficient_schedulers.items()}

    @torch.no_grad()
    def _build_train_step_log_dict(self, output: TrainStepOutput, n_training_samples: int) -> dict[str, Any]:
        sae_in, sae_out = output.sae_in.float(), output.sae_out.float()
        fa = output.feature_acts
        l0 = fa.l0() if isinstance(fa, _LazySparse) else fa.bool().float().sum(-1).to_dense().mean()
        per_tok = (sae_out - sae_in).pow(2).sum(dim=-1).squeeze()
        tot_var = (sae_in - sae_in.mean(0)).pow(2).sum(-1)
        ev_legacy = 1 - per_tok / tot_var
        ev = 1 - per_tok.mean() / tot_var.mean()
        d = {
            "losses/overall_loss": output.loss.item(),
            "metrics/explained_variance_legacy": ev_legacy.mean().item(),
            "metrics/explained_variance_legacy_std": ev_legacy.std().item(),
            "metrics/explained_variance": ev.item(),
            "metrics/l0": float(l0),
            "sparsity/mean_passes_since_fired": self.n_forward_passes_since_fired.mean().item(),
            "sparsity/dead_features": self.dead_neurons.sum().item(),
            "details/current_learning_rate": self.current_lr(),
            "details/n_training_samples": n_training_samples,
            **{f"details/{n}_coefficient": s.value for n, s in self.coefficient_schedulers.items()},
        }
        for n, v in output.losses.items():
            d[f"losses/{n}"] = _unwrap_item(v)
        for n, v in output.metrics.items():
            d[f"metrics/{n}"] = _unwrap_item(v)
        return d

    @torch.no_grad()
    def _run_and_log_evals(self) -> None:
        every = self.cfg.logger.wandb_log_frequency * self.cfg.logger.eval_every_n_wandb_logs
        if (self.n_training_steps + 1) % every != 0:
            return
        if self._native_fsdp:  # the module holds one latent shard until the end of training
            if not self._warned_fsdp_evals:
                logger.warning("evals are skipped during sharded data-parallel training on the native engine")
                self._warned_fsdp_evals = True
            return
        self.sae.eval()
        metrics = self.evaluator(self._base_sae, self.data_provider, self.activation_scaler) if self.evaluator else {}
        for k, v in self._base_sae.log_histograms().items():
            metrics[k] = wandb.Histogram(v)
        wandb.log(metrics, step=self.n_training_steps)
        self.sae.train()

    @torch.no_grad()
    def _build_sparsity_log_dict(self) -> dict[str, Any]:
        lfs = _log_feature_sparsity(self.feature_sparsity)
        return {"metrics/mean_log10_feature_sparsity": lfs.mean().item(),
                "plots/feature_density_line_chart": wandb.Histogram(lfs.numpy()),
                "sparsity/below_1e-5": (self.feature_sparsity < 1e-5).sum().item(),
                "sparsity/below_1e-6": (self.feature_sparsity < 1e-6).sum().item()}

    @torch.no_grad()
    def _reset_running_sparsity_stats(self) -> None:
        self.act_freq_scores = torch.zeros_like(self.act_freq_scores)
        self.n_frac_active_samples = 0

    @torch.no_grad()
    def _checkpoint_if_needed(self) -> None:
        if self.checkpoint_thresholds and self.n_training_samples > self.checkpoint_thresholds[0]:
            self.save_checkpoint(checkpoint_name=str(self.n_training_samples))
            self.checkpoint_thresholds.pop(0)


class _LazySparse:
    """Feature activations of a native step: materialised (sparse COO) only on request."""

    def __init__(self, res: Any, d_sae: int):
        self._res, self._d = res, d_sae

    def l0(self) -> float:
        r = self._res
        if r.topk_idx is None:
            return float(r.l0)
        return float(((r.topk_idx >= 0) & (r.topk_vals > 0)).sum(-1).float().mean())

    def to_sparse(self) -> torch.Tensor:
        return self._res.feature_acts_sparse(self._d)

    def bool(self) -> torch.Tensor:
        return self.to_sparse().bool()

    def to_dense(self) -> torch.Tensor:
        return self.to_sparse().to_dense()
