"""`LanguageModelSAETrainingRunner`: train an SAE on a language model's activations end to end
(API of sae_lens/llm_sae_training_runner.py).

run(): process groups (when launched with torchrun) -> producer LM -> ActivationsStore ->
TrainingSAE (optionally sharded over `sae_tp_size` ranks, replicated over `sae_dp_size` ranks
with manual / DDP / FSDP gradient sync) -> SAETrainer.fit() -> final inference SAE, feature
sparsity and `runner_cfg.json`.  On CUDA, TopK SAEs train on the fused native engine.
SIGINT/SIGTERM checkpoint the run before exiting.

Command line: `python -m saelens_b200.runners.llm_sae_training_runner --architecture topk --d_in ...`
(every config field is a `--field value` flag; nested SAE fields are plain flags too).
"""

from __future__ import annotations

import json
import os
from datetime import timedelta
import signal
import sys
from dataclasses import fields
from pathlib import Path
from typing import Any

import torch
import torch.distributed as dist

from saelens_b200 import logger
from saelens_b200.config import LanguageModelSAERunnerConfig, LoggingConfig
from saelens_b200.constants import (
    ACTIVATIONS_STORE_STATE_FILENAME,
    RUNNER_CFG_FILENAME,
    SAE_WEIGHTS_FILENAME,
    SPARSITY_FILENAME,
)
from saelens_b200.models.sae import TrainingSAE, TrainingSAEConfig
from saelens_b200.registry import get_sae_training_class
from saelens_b200.training.activations_store import ActivationsStore
from saelens_b200.training.sae_trainer import SAETrainer


class InterruptedException(Exception):
    pass


def _interrupt(*_a: Any) -> None:
    raise InterruptedException()


class LanguageModelSAETrainingRunner:
    def __init__(self, cfg: LanguageModelSAERunnerConfig[Any], override_dataset: Any = None,
                 override_model: Any = None, override_sae: TrainingSAE[Any] | None = None,
                 resume_from_checkpoint: str | Path | None = None, sae_tp_size: int = 1, sae_dp_size: int = 1,
                 vllm_tp_size: int = 1, vllm_dp_size: int = 1, use_shard_routing: bool = False,
                 streaming_mode: bool | None = None, token_count_weighted_dp: bool = False):
        self.cfg = cfg
        self.override_dataset = override_dataset
        self.override_model = override_model
        self.override_sae = override_sae
        self.resume_from_checkpoint = resume_from_checkpoint or cfg.resume_from_checkpoint
        self.sae_tp_size, self.sae_dp_size = sae_tp_size, sae_dp_size
        self.vllm_tp_size, self.vllm_dp_size = vllm_tp_size, vllm_dp_size
        self.use_shard_routing = use_shard_routing
        self.streaming_mode = cfg.streaming_mode if streaming_mode is None else streaming_mode
        self.token_count_weighted_dp = token_count_weighted_dp
        self.tp_group: dist.ProcessGroup | None = None
        self.dp_group: dist.ProcessGroup | None = None
        self.ddp_hook_state: Any = None  # P2P gradient all-reduce of the DDP wrapper, when used
        self.native_fsdp = False  # sae_dp_mode="fsdp" on the native sharded engine
        self.role: str | None = None  # streaming / routed mode: producer (LM), consumer (SAE) or both
        self.router: Any = None
        self.routed = bool(use_shard_routing) and int(os.environ.get("WORLD_SIZE", "1")) > 1 and not self.streaming_mode
        if self.streaming_mode:
            from saelens_b200.runners.streaming import streaming_init

            streaming_init(self)  # groups, roles and the activation ring (collective)
        elif self.routed:
            from saelens_b200.runners.routing import routing_init

            routing_init(self)  # v2 layout, roles and the row router (collective)
        else:
            self._init_distributed()
        self._sync_run_paths_across_ranks()
        self.fan_in = False
        if not (self.streaming_mode or self.routed) and dist.is_available() and dist.is_initialized():
            from saelens_b200.parallel import distributed as D

            if D.get_layout_mode() == "vllm_dp_fan_in":  # legacy m:1 / mn:m producers -> SAE roots
                if self.sae_tp_size > 1:
                    raise ValueError("the fan-in data path serves SAE TP 1; use shard routing for TP consumers")
                self.fan_in = True
                self.role = "producer+consumer" if D.is_sae_active() else "producer"
        # split roles (local overlap / matched DP with SAE TP): only the replica's LM root runs the LM
        # and broadcasts each batch to its SAE TP group (sae_lens/training/activations_store.py:617-738)
        self.split_role = False
        if not (self.streaming_mode or self.routed or self.fan_in) and self.tp_group is not None:
            from saelens_b200.parallel import distributed as D

            if D.get_layout_mode() in ("local_overlap", "matched_dp"):
                self.split_role = True
                self.role = "producer+consumer" if D.get_worker_rank() == 0 else "consumer"
        if self.routed:
            producer_side, consumer_side = self.is_route_producer, self.is_route_consumer
        elif self.split_role:
            producer_side, consumer_side = self.role == "producer+consumer", True
        elif self.fan_in:
            producer_side, consumer_side = True, self.role == "producer+consumer"
        else:
            producer_side = self.role in (None, "producer")
            consumer_side = self.role in (None, "consumer")
        self.model = None
        self.activations_store: Any = None
        if producer_side:
            self.model = override_model if override_model is not None else self._load_model()
            if getattr(self, "producer_tp_group", None) is not None:
                from saelens_b200.models.lm.tp import shard_lm_tensor_parallel

                shard_lm_tensor_parallel(self.model, self.producer_tp_group)  # Megatron split of the producer
            if cfg.compile_llm:
                self.model = torch.compile(self.model, mode=cfg.llm_compilation_mode)
            if self.streaming_mode:
                shard, nshard = self._streaming_producer_shard()
            elif self.routed:
                from saelens_b200.parallel import distributed_v2 as v2

                n = max(self.vllm_dp_size, 1)
                shard, nshard = (v2.get_producer_idx(), n) if n > 1 else (0, 1)
            elif self.fan_in:
                from saelens_b200.parallel import distributed as D

                shard, nshard = D.get_vllm_dp_rank(), max(self.vllm_dp_size, 1)
            else:
                shard, nshard = (self._dp_rank(), self.sae_dp_size) if self.sae_dp_size > 1 else (0, 1)
            self.activations_store = ActivationsStore.from_config(self.model, cfg, override_dataset=override_dataset,
                                                                  shard_index=shard, num_shards=nshard)
        self.sae: Any = None
        self.wrapped: Any = None
        self.hook_names = list(cfg.hook_names) if cfg.hook_names else [cfg.hook_name]
        self.is_multi_sae = len(self.hook_names) > 1
        self.sae_by_hook: dict[str, Any] = {}
        self.base_sae_by_hook: dict[str, Any] = {}
        if consumer_side and self.is_multi_sae:
            self._init_multi_saes()
        elif consumer_side:
            self.sae = override_sae if override_sae is not None else self._build_sae()
            if self.tp_group is not None and hasattr(self.sae, "shard_weights"):
                self.sae.shard_weights(self.tp_group)
            self._compile_sae_if_needed(self.sae)
            self.wrapped = self._wrap_dp(self.sae)

    # ---------------------------------------------------------------- setup
    def _streaming_producer_shard(self) -> tuple[int, int]:
        """Each streaming producer reads its own slice of the token dataset."""
        from saelens_b200.parallel import distributed_streaming as ds

        n = max(self.vllm_dp_size, 1)
        return (ds.get_producer_idx(), n) if n > 1 else (0, 1)

    def _init_distributed(self) -> None:
        world = int(os.environ.get("WORLD_SIZE", "1"))
        single_layout = (self.sae_tp_size == 1 and self.sae_dp_size == 1 and self.vllm_dp_size <= 1
                         and self.vllm_tp_size <= 1)
        if world <= 1 or (single_layout and not self.use_shard_routing and not self.streaming_mode):
            return
        if not dist.is_initialized():
            backend = "nccl" if self.cfg.device.startswith("cuda") else "gloo"
            kw: dict[str, Any] = {}
            if backend == "nccl":
                local = int(os.environ.get("LOCAL_RANK", "0"))
                torch.cuda.set_device(local)
                kw["device_id"] = torch.device("cuda", local)
            # a short collective timeout: ranks left waiting on a rank that failed end with an error
            kw["timeout"] = timedelta(seconds=float(os.environ.get("SAELENS_B200_PG_TIMEOUT_S", "300")))
            dist.init_process_group(backend, **kw)
        from saelens_b200.parallel import distributed as D

        D.init_distributed(sae_tp_size=self.sae_tp_size, sae_dp_size=self.sae_dp_size,
                           vllm_tp_size=max(self.vllm_tp_size, 1), vllm_dp_size=max(self.vllm_dp_size, self.sae_dp_size))
        self.tp_group = D.get_sae_tp_group() if self.sae_tp_size > 1 else None
        self.dp_group = D.get_sae_dp_group() if self.sae_dp_size > 1 else None

    def _dp_rank(self) -> int:
        return dist.get_rank(self.dp_group) if self.dp_group is not None else 0

    def _load_model(self) -> Any:
        from saelens_b200.models.lm.load_model import load_model

        return load_model(self.cfg.model_class_name, self.cfg.model_name, device=self.cfg.device,
                          model_from_pretrained_kwargs=self.cfg.model_from_pretrained_kwargs)

    def _build_sae(self) -> TrainingSAE[Any]:
        cfg = self.cfg
        if cfg.from_pretrained_path is not None:
            sae = TrainingSAE.load_from_disk(cfg.from_pretrained_path, device=cfg.device)
        else:
            sae_cfg = type(cfg.sae).from_sae_runner_config(cfg)
            sae_cfg.device = cfg.device
            sae_cfg.dtype = cfg.dtype
            torch.manual_seed(cfg.seed)
            sae = get_sae_training_class(sae_cfg.architecture())[0](sae_cfg)
        return sae

    def _sync_run_paths_across_ranks(self) -> None:
        """Every rank uses rank 0's output and checkpoint paths (default paths carry a timestamp,
        which differs between processes started a second apart)."""
        if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
            return
        paths = [self.cfg.output_path, self.cfg.checkpoint_path]
        dist.broadcast_object_list(paths, src=0)
        self.cfg.output_path, self.cfg.checkpoint_path = paths

    def _compile_sae_if_needed(self, sae: Any) -> None:
        """`compile_sae`: compile the SAE's training forward before any DP wrapping (the PyTorch
        path; the native engines do not run it)."""
        if self.cfg.compile_sae:
            sae.training_forward_pass = torch.compile(sae.training_forward_pass, mode=self.cfg.sae_compilation_mode)

    def _init_multi_saes(self) -> None:
        """One SAE per hook, trained from one LM pass (sae_lens/llm_sae_training_runner.py:489-584):
        the same seed for every hook ("same") or seed + index ("offset"); each SAE records its hook
        in the metadata, is sharded for TP and wrapped for DDP / FSDP like a single SAE."""
        cfg = self.cfg
        for idx, hook in enumerate(self.hook_names):
            seed = cfg.seed if cfg.multi_sae_seed_mode == "same" else cfg.seed + idx
            sae_cfg = type(cfg.sae).from_sae_runner_config(cfg)
            sae_cfg.device = cfg.device
            sae_cfg.dtype = cfg.dtype
            from saelens_b200.utils.misc import temporary_seed

            with temporary_seed(seed):  # the global RNG stream is left as it was
                sae = get_sae_training_class(sae_cfg.architecture())[0](sae_cfg)
            sae.cfg.metadata.hook_name = hook
            if self.tp_group is not None and hasattr(sae, "shard_weights"):
                sae.shard_weights(self.tp_group)
            self._compile_sae_if_needed(sae)
            self.base_sae_by_hook[hook] = sae
            if self.dp_group is not None and cfg.sae_dp_mode == "fsdp":
                from torch.distributed.fsdp import FullyShardedDataParallel as FSDP
                from torch.distributed.fsdp import ShardingStrategy

                self.sae_by_hook[hook] = FSDP(sae, process_group=self.dp_group,
                                              sharding_strategy=ShardingStrategy.FULL_SHARD, use_orig_params=True,
                                              device_id=sae.W_dec.device if sae.W_dec.is_cuda else None)
            elif self.dp_group is not None and cfg.sae_dp_mode == "ddp":
                from torch.nn.parallel import DistributedDataParallel as DDP

                kw: dict[str, Any] = {"process_group": self.dp_group}
                if sae.W_dec.is_cuda:
                    kw["device_ids"] = [sae.W_dec.device.index]
                self.sae_by_hook[hook] = DDP(sae, **kw)
            else:
                self.sae_by_hook[hook] = sae

    def _run_multi(self) -> dict[str, Any]:
        from saelens_b200.training.multi_sae_trainer import MultiSAETrainer

        cfg = self.cfg
        trainer = MultiSAETrainer(
            hook_names=self.hook_names, sae_by_hook=self.sae_by_hook, base_sae_by_hook=self.base_sae_by_hook,
            data_provider=self.activations_store, cfg=cfg.to_sae_trainer_config(), dp_group=self.dp_group,
            token_count_weighted_dp=self.token_count_weighted_dp, sae_dp_mode=cfg.sae_dp_mode,
            backward_mode=cfg.multi_sae_backward_mode, seed_mode=cfg.multi_sae_seed_mode)
        self.trainer = trainer
        if self.resume_from_checkpoint is not None:
            trainer.load_trainer_state(self.resume_from_checkpoint)
            if (Path(self.resume_from_checkpoint) / ACTIVATIONS_STORE_STATE_FILENAME).exists():
                self.activations_store.load_from_checkpoint(self.resume_from_checkpoint)
        result = trainer.fit()
        if cfg.output_path is not None:
            trainer.save_final(cfg.output_path)  # every rank (TP gathers are collective); one writes
            if self._is_writer():
                with open(Path(cfg.output_path) / RUNNER_CFG_FILENAME, "w") as f:
                    json.dump(cfg.to_dict(), f, default=str)
        return result

    def _native_fsdp_ok(self, sae: TrainingSAE[Any]) -> bool:
        """TopK / BatchTopK / JumpReLU on CUDA with the native ops, at most 8 NCCL ranks (one
        NVSwitch domain), d_sae divisible into 256-latent tiles per rank."""
        if self.cfg.sae_engine == "torch" or not sae.W_dec.is_cuda:
            return False
        from saelens_b200.parallel.fsdp_jumprelu_engine import fsdp_jumprelu_supported
        from saelens_b200.training.engine import engine_supported

        world = dist.get_world_size(self.dp_group)
        if not (1 < world <= 8 and dist.get_backend(self.dp_group) == "nccl"):
            return False
        return ((engine_supported(sae) and sae.W_dec.shape[0] % (256 * world) == 0)
                or fsdp_jumprelu_supported(sae, world))

    def _wrap_dp(self, sae: TrainingSAE[Any]) -> Any:
        if self.dp_group is None or self.cfg.sae_dp_mode == "manual":
            return sae
        if self.cfg.sae_dp_mode == "ddp":
            from torch.nn.parallel import DistributedDataParallel as DDP

            kw: dict[str, Any] = {"process_group": self.dp_group}
            for k in ("broadcast_buffers", "find_unused_parameters", "gradient_as_bucket_view", "static_graph",
                      "bucket_cap_mb"):
                v = getattr(self.cfg, f"ddp_{k}")
                if v is not None:
                    kw[k] = v
            if sae.W_dec.is_cuda:
                kw["device_ids"] = [sae.W_dec.device.index]
            ddp = DDP(sae, **kw)
            if getattr(self.cfg, "ddp_exchange", "p2p") == "p2p":
                from saelens_b200.parallel.p2p_ddp_hook import p2p_hook_supported, register_p2p_allreduce

                if p2p_hook_supported(sae, self.dp_group):
                    self.ddp_hook_state = register_p2p_allreduce(ddp, sae, self.dp_group, kw.get("bucket_cap_mb"))
            return ddp
        if self.tp_group is not None:
            raise ValueError("sae_dp_mode='fsdp' cannot be combined with sae_tp_size > 1")
        if self._native_fsdp_ok(sae):
            self.native_fsdp = True  # the trainer's FSDPTopKEngine shards the module itself
            return sae
        from torch.distributed.fsdp import FullyShardedDataParallel as FSDP
        from torch.distributed.fsdp import ShardingStrategy

        return FSDP(sae, process_group=self.dp_group, sharding_strategy=ShardingStrategy.FULL_SHARD,
                    use_orig_params=True, device_id=sae.W_dec.device if sae.W_dec.is_cuda else None)

    # ---------------------------------------------------------------- run
    def run(self) -> TrainingSAE[Any]:
        cfg = self.cfg
        if self.streaming_mode:
            from saelens_b200.runners.streaming import run_streaming

            return run_streaming(self)
        if self.routed:
            return self._run_routed()
        if self.is_multi_sae:
            return self._run_multi()
        if self.fan_in:
            return self._run_fan_in()
        return self._run_standard()

    def _run_fan_in(self) -> Any:
        """Fan-in: helpers serve activation batches to their cluster's SAE root."""
        from saelens_b200.parallel import distributed as D
        from saelens_b200.runners.fan_in import FanInRoot, run_helper

        group = D.get_vllm_dp_p2p_group()
        root = D.get_sae_root_rank()
        sae = None
        if self.role == "producer":
            run_helper(self.activations_store, root, group)
        else:
            block = D.get_cluster_block()
            fan = FanInRoot(self.activations_store, [root + i for i in range(1, block)], group)
            try:
                sae = self._run_standard()
            finally:
                fan.close()
        dist.barrier()
        return sae

    def _run_standard(self) -> Any:
        cfg = self.cfg
        if cfg.logger.log_to_wandb and self._is_writer():
            from saelens_b200.utils import wandb_shim as wandb

            wandb.init(project=cfg.logger.wandb_project, entity=cfg.logger.wandb_entity, name=cfg.logger.run_name,
                       id=cfg.logger.wandb_id, config=cfg.to_dict())
        data: Any = self.activations_store
        if self.split_role:
            from saelens_b200.parallel import distributed as D
            from saelens_b200.training.replica_broadcast import ReplicaBroadcastProvider
            from saelens_b200.utils.misc import str_to_dtype

            data = ReplicaBroadcastProvider(self.activations_store, self.tp_group, D.get_sae_root_rank(),
                                            self.sae.cfg.d_in, str_to_dtype(cfg.dtype), cfg.act_store_device)
        trainer = SAETrainer(
            cfg=cfg.to_sae_trainer_config(), sae=self.wrapped, base_sae=self.sae, data_provider=data,
            evaluator=self._evaluator() if self.activations_store is not None else None,
            save_checkpoint_fn=self._save_checkpoint_extras, dp_group=self.dp_group,
            token_count_weighted_dp=self.token_count_weighted_dp, native_fsdp=self.native_fsdp,
            append_logs=self.resume_from_checkpoint is not None,  # a resumed run continues its histories
        )
        self.trainer = trainer
        if self.resume_from_checkpoint is not None:
            ck = Path(self.resume_from_checkpoint)
            if self.native_fsdp:
                # the module holds one latent shard: the engine takes its part of the full weights
                from safetensors.torch import load_file

                sd = load_file(ck / SAE_WEIGHTS_FILENAME)
                self.sae.process_state_dict_for_loading(sd)
                trainer.engine.load_weights(sd["W_enc"], sd["W_dec"], sd["b_enc"], sd["b_dec"])
                if "topk_threshold" in sd and hasattr(self.sae, "topk_threshold"):
                    self.sae.topk_threshold.copy_(sd["topk_threshold"])
            else:
                self.sae.load_weights_from_checkpoint(ck)
            if trainer.engine is not None and not self.native_fsdp:
                trainer.engine.refresh()
            trainer.load_trainer_state(ck)
            if (ck / ACTIVATIONS_STORE_STATE_FILENAME).exists() and self.activations_store is not None:
                self.activations_store.load_from_checkpoint(ck)
        old_int = signal.signal(signal.SIGINT, _interrupt)
        old_term = signal.signal(signal.SIGTERM, _interrupt)
        try:
            sae = trainer.fit()
            if self.ddp_hook_state is not None:
                self.ddp_hook_state.check()
        except (KeyboardInterrupt, InterruptedException):
            logger.warning("interrupted: saving a checkpoint before exiting")
            trainer.save_checkpoint(checkpoint_name=f"interrupted_{trainer.n_training_samples}")
            raise
        finally:
            signal.signal(signal.SIGINT, old_int)
            signal.signal(signal.SIGTERM, old_term)
        self.save_final_sae(sae, trainer)
        if cfg.logger.log_to_wandb and self._is_writer():
            from saelens_b200.utils import wandb_shim as wandb

            wandb.finish()
        return sae

    def _run_routed(self) -> Any:
        """Shard-routing mode: producers feed the consumers' trainers step by step."""
        from saelens_b200.runners.routing import RoutedExchange, RoutedProvider, resume_state, run_producer_only

        cfg = self.cfg
        n_steps = cfg.total_training_steps
        sae = None
        if not self.is_route_consumer:
            run_producer_only(self, n_steps)
        elif self.is_multi_sae:
            sae = self._run_routed_multi(n_steps)
        else:
            ex = RoutedExchange(self)
            done = resume_state(self, ex)
            trainer = SAETrainer(
                cfg=cfg.to_sae_trainer_config(), sae=self.wrapped, base_sae=self.sae,
                data_provider=RoutedProvider(ex, n_steps - done), evaluator=None,
                save_checkpoint_fn=self._save_checkpoint_extras if self.activations_store is not None else None,
                dp_group=self.dp_group, native_fsdp=self.native_fsdp,
                append_logs=self.resume_from_checkpoint is not None)
            self.trainer = trainer
            if self.resume_from_checkpoint is not None:
                ck = Path(self.resume_from_checkpoint)
                self.sae.load_weights_from_checkpoint(ck)
                if trainer.engine is not None:
                    trainer.engine.refresh()
                trainer.load_trainer_state(ck)
            sae = trainer.fit()
            ex.finish()
            self.save_final_sae(sae, trainer)
        dist.barrier()
        if self.router is not None:
            self.router.close()
        return sae

    def _run_routed_multi(self, n_steps: int) -> Any:
        """Routed consumer with one SAE per hook: each routed step's rows carry every hook, and
        `MultiSAETrainer` trains the hooks' SAEs on them (data parallel over the consumers)."""
        from saelens_b200.runners.routing import RoutedExchange, RoutedProvider, resume_state
        from saelens_b200.training.multi_sae_trainer import MultiSAETrainer

        cfg = self.cfg
        ex = RoutedExchange(self)
        done = resume_state(self, ex)
        trainer = MultiSAETrainer(
            hook_names=self.hook_names, sae_by_hook=self.sae_by_hook, base_sae_by_hook=self.base_sae_by_hook,
            data_provider=RoutedProvider(ex, n_steps - done, self.hook_names), cfg=cfg.to_sae_trainer_config(),
            dp_group=self.dp_group, token_count_weighted_dp=self.token_count_weighted_dp,
            sae_dp_mode=cfg.sae_dp_mode, backward_mode=cfg.multi_sae_backward_mode,
            seed_mode=cfg.multi_sae_seed_mode)
        self.trainer = trainer
        if self.resume_from_checkpoint is not None:
            trainer.load_trainer_state(self.resume_from_checkpoint)
        result = trainer.fit()
        ex.finish()
        if cfg.output_path is not None:
            trainer.save_final(cfg.output_path)  # every consumer rank (TP gathers); the first writes
        return result

    def _evaluator(self) -> Any:
        from saelens_b200.evals import LLMSaeEvaluator

        return LLMSaeEvaluator(self.model, self.activations_store, self.cfg.n_eval_batches,
                               self.cfg.eval_batch_size_prompts)

    def _is_writer(self) -> bool:
        tp = dist.get_rank(self.tp_group) if self.tp_group is not None else 0
        dp = dist.get_rank(self.dp_group) if self.dp_group is not None else 0
        return tp == 0 and dp == 0

    def _save_checkpoint_extras(self, checkpoint_path: Path | None) -> None:
        if checkpoint_path is None or self.activations_store is None:
            return
        self.activations_store.save_to_checkpoint(checkpoint_path)
        with open(Path(checkpoint_path) / RUNNER_CFG_FILENAME, "w") as f:
            json.dump(self.cfg.to_dict(), f, default=str)

    def save_final_sae(self, sae: TrainingSAE[Any], trainer: SAETrainer[Any]) -> Path | None:
        if self.cfg.output_path is None:
            return None
        out = Path(self.cfg.output_path)
        out.mkdir(parents=True, exist_ok=True)
        sae.save_inference_model(out)
        if self._is_writer():
            from safetensors.torch import save_file

            save_file({"sparsity": trainer.log_feature_sparsity}, out / SPARSITY_FILENAME)
            with open(out / RUNNER_CFG_FILENAME, "w") as f:
                json.dump(self.cfg.to_dict(), f, default=str)
        return out


SAETrainingRunner = LanguageModelSAETrainingRunner


# ------------------------------------------------------------------------------ CLI
def _coerce(tp: Any, raw: str) -> Any:
    s = str(tp)
    if raw.lower() in ("none", "null") and ("None" in s or "Optional" in s):
        return None
    if "bool" in s and raw.lower() in ("true", "false", "1", "0", "yes", "no"):
        return raw.lower() in ("true", "1", "yes")
    if s.startswith("dict") or "dict[" in s:
        return json.loads(raw)
    if "tuple" in s:
        return tuple(None if x in ("", "None") else int(x) for x in raw.strip("()").split(",") if x.strip() != "" or True)
    if "list[int]" in s and raw.startswith("["):
        return json.loads(raw)
    if "int" in s and "float" not in s and "str" not in s:
        try:
            return int(raw)
        except ValueError:
            pass
    if "float" in s:
        try:
            return float(raw)
        except ValueError:
            pass
    if "int" in s:
        try:
            return int(raw)
        except ValueError:
            pass
    return raw


def _parse_cfg_args(args: list[str]) -> LanguageModelSAERunnerConfig[Any]:
    """`--architecture <arch>` selects the SAE training config; every other `--field value` is a
    runner, logger or SAE config field."""
    kv: dict[str, str] = {}
    i = 0
    while i < len(args):
        a = args[i]
        if not a.startswith("--"):
            raise SystemExit(f"unexpected argument {a!r}")
        key = a[2:].replace("-", "_")
        if "=" in key:
            key, val = key.split("=", 1)
            i += 1
        elif i + 1 < len(args) and not args[i + 1].startswith("--"):
            val = args[i + 1]
            i += 2
        else:
            val = "true"
            i += 1
        kv[key] = val
    arch = kv.pop("architecture", "standard")
    sae_cfg_cls = get_sae_training_class(arch)[1]
    sae_f = {f.name: f.type for f in fields(sae_cfg_cls)}
    run_f = {f.name: f.type for f in fields(LanguageModelSAERunnerConfig)}
    log_f = {f.name: f.type for f in fields(LoggingConfig)}
    sae_kw, run_kw, log_kw = {}, {}, {}
    for k, v in kv.items():
        if k in sae_f and k not in ("device", "dtype"):
            sae_kw[k] = _coerce(sae_f[k], v)
        elif k in run_f:
            run_kw[k] = _coerce(run_f[k], v)
        elif k in log_f:
            log_kw[k] = _coerce(log_f[k], v)
        elif k in sae_f:
            sae_kw[k] = _coerce(sae_f[k], v)
        else:
            raise SystemExit(f"unknown option --{k}")
    if "d_in" not in sae_kw or "d_sae" not in sae_kw:
        raise SystemExit("--d_in and --d_sae are required")
    sae_cfg: TrainingSAEConfig = sae_cfg_cls(**sae_kw)
    return LanguageModelSAERunnerConfig(sae=sae_cfg, logger=LoggingConfig(**log_kw), **run_kw)


def _run_cli(args: list[str]) -> None:
    cfg = _parse_cfg_args(args)
    LanguageModelSAETrainingRunner(cfg).run()


if __name__ == "__main__":
    _run_cli(sys.argv[1:])
