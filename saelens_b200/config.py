"""Run configurations: field names and defaults of the reference (sae_lens/config.py), as plain
dataclasses (the command line is parsed by `saelens_b200.runners.cli`)."""

from __future__ import annotations

import json
import logging
import math
import warnings
from dataclasses import asdict, dataclass, field
from datetime import datetime
from pathlib import Path
from typing import Any, Generic, Literal, TypeVar

import torch

from saelens_b200 import __version__
from saelens_b200.models.sae import TrainingSAEConfig
from saelens_b200.registry import get_sae_training_class
from saelens_b200.utils.misc import str_to_dtype

logger = logging.getLogger("saelens_b200")

T_TRAINING_SAE_CONFIG = TypeVar("T_TRAINING_SAE_CONFIG", bound=TrainingSAEConfig)

SpecialToken = int | Literal["bos", "eos", "sep"] | None


def _timestamp_run_id() -> str:
    return datetime.now().strftime("%y%m%d_%H%M%S")


def _unique_run_id(base: Path, run_id: str) -> str:
    cand, i = run_id, 1
    while (base / cand).exists():
        cand = f"{run_id}_{i}"
        i += 1
    return cand


def json_dict(s: str) -> Any:
    res = json.loads(s)
    if res is not None and not isinstance(res, dict):
        raise ValueError(f"Expected a dictionary, got {type(res)}")
    return res


def special_token(s: str) -> SpecialToken:
    if s.lower() == "none":
        return None
    if s in ("bos", "eos", "sep"):
        return s  # type: ignore[return-value]
    try:
        return int(s)
    except ValueError as e:
        raise ValueError(f"Expected 'bos', 'eos', 'sep', an integer, or 'none', got {s}") from e


@dataclass
class LoggingConfig:
    log_to_wandb: bool = True
    log_activations_store_to_wandb: bool = False
    log_optimizer_state_to_wandb: bool = False
    log_weights_to_wandb: bool = True
    wandb_project: str = "sae_lens_training"
    wandb_id: str | None = None
    run_name: str | None = None
    wandb_entity: str | None = None
    wandb_log_frequency: int = 10
    eval_every_n_wandb_logs: int = 100

    def log(self, trainer: Any, weights_path: Path | str, cfg_path: Path | str,
            sparsity_path: Path | str | None, wandb_aliases: list[str] | None = None) -> None:
        from saelens_b200.utils import wandb_shim as wandb

        name = trainer.sae.get_name().replace("/", "__")
        art = wandb.Artifact(name, type="model", metadata=dict(trainer.cfg.__dict__))
        if self.log_weights_to_wandb:
            art.add_file(str(weights_path))
        art.add_file(str(cfg_path))
        wandb.log_artifact(art, aliases=wandb_aliases)
        sp = wandb.Artifact(f"{name}_log_feature_sparsity", type="log_feature_sparsity",
                            metadata=dict(trainer.cfg.__dict__))
        if sparsity_path is not None:
            sp.add_file(str(sparsity_path))
        wandb.log_artifact(sp)


def _validate_seqpos(seqpos: tuple[int | None, ...], context_size: int) -> None:
    if len(seqpos) == 3:
        step = seqpos[2] or 1
        if step <= 1:
            raise ValueError(f"Ensure the step_size={seqpos[2]} for sequence slicing is at least 1.")
    if len(list(range(context_size))[slice(*seqpos)]) == 0:
        raise ValueError(f"The slice {seqpos} results in an empty range. Please adjust your seqpos or context_size.")


def _default_cached_activations_path(dataset_path: str, model_name: str, hook_name: str,
                                     hook_head_index: int | None) -> str:
    p = f"activations/{dataset_path.replace('/', '_')}/{model_name.replace('/', '_')}/{hook_name}"
    if hook_head_index is not None:
        p += f"_{hook_head_index}"
    return p


@dataclass
class LanguageModelSAERunnerConfig(Generic[T_TRAINING_SAE_CONFIG]):
    """Configuration for training an SAE on a language model's activations.

    Field names, meanings and defaults follow the reference runner config
    (sae_lens/config.py:142-506), including the fork's DP/DDP/multi-SAE/streaming knobs.
    """

    sae: T_TRAINING_SAE_CONFIG

    model_name: str = "gelu-2l"
    model_class_name: str = "HookedTransformer"
    hook_name: str = "blocks.0.hook_mlp_out"
    hook_names: list[str] | None = None
    hook_eval: str = "NOT_IN_USE"
    hook_head_index: int | None = None
    dataset_path: str = ""
    dataset_trust_remote_code: bool = True
    streaming: bool = True
    is_dataset_tokenized: bool = True
    context_size: int = 128
    use_cached_activations: bool = False
    cached_activations_path: str | None = None

    from_pretrained_path: str | None = None

    n_batches_in_buffer: int = 20
    training_tokens: int = 2_000_000
    store_batch_size_prompts: int = 32
    seqpos_slice: tuple[int | None, ...] = (None,)
    disable_concat_sequences: bool = False
    sequence_separator_token: SpecialToken = "bos"
    activations_mixing_fraction: float = 0.5

    device: str = "cpu"
    act_store_device: str = "with_model"
    seed: int = 42
    dtype: str = "float32"
    prepend_bos: bool = True

    autocast: bool = False
    autocast_lm: bool = False
    compile_llm: bool = False
    llm_compilation_mode: str | None = None
    compile_sae: bool = False
    sae_compilation_mode: str | None = None

    train_batch_size_tokens: int = 4096

    adam_beta1: float = 0.9
    adam_beta2: float = 0.999

    lr: float = 3e-4
    lr_scheduler_name: str = "constant"
    lr_warm_up_steps: int = 0
    lr_end: float | None = None
    lr_decay_steps: int = 0
    n_restart_cycles: int = 1

    dead_feature_window: int = 1000
    feature_sampling_window: int = 2000
    dead_feature_threshold: float = 1e-8

    n_eval_batches: int = 10
    eval_batch_size_prompts: int | None = None

    logger: LoggingConfig = field(default_factory=LoggingConfig)

    n_checkpoints: int = 0
    checkpoint_path: str | None = "checkpoints"
    save_final_checkpoint: bool = False
    output_path: str | None = "output"
    save_mse_every_n_steps: int = 0
    save_timing_every_n_steps: int = 0
    save_memory_every_n_steps: int = 0
    synchronize_timing: bool = False
    resume_from_checkpoint: str | None = None

    verbose: bool = True
    model_kwargs: dict[str, Any] = field(default_factory=dict)
    model_from_pretrained_kwargs: dict[str, Any] | None = None
    sae_lens_version: str = field(default_factory=lambda: __version__)
    sae_lens_training_version: str = field(default_factory=lambda: __version__)
    exclude_special_tokens: bool | list[int] = False
    sae_dp_mode: Literal["manual", "ddp", "fsdp"] = "manual"
    multi_sae_backward_mode: Literal["combined", "sequential"] = "combined"
    multi_sae_backward_order: Literal["forward", "reverse", "largest_first"] = "forward"
    multi_sae_stats_sync_mode: Literal["immediate", "deferred", "periodic"] = "immediate"
    multi_sae_stats_sync_interval: int = 1
    multi_sae_seed_mode: Literal["same", "offset"] = "same"
    ddp_broadcast_buffers: bool | None = None
    ddp_find_unused_parameters: bool | None = None
    ddp_gradient_as_bucket_view: bool | None = None
    ddp_static_graph: bool | None = None
    ddp_bucket_cap_mb: int | None = None
    ddp_config_strict: bool = False

    streaming_mode: bool = False
    streaming_chunk_size_tokens: int = 4096
    streaming_num_chunks: int = 32
    streaming_prefetch_chunks: int = 2
    streaming_buffer_name: str = ""
    streaming_shuffle: bool = True
    streaming_random_chunks: bool = True
    # Transport of streaming mode (no counterpart in the reference): "device" = ring in the
    # consumer GPU's memory written over NVLink, "host" = the /dev/shm ring, "auto" = device when
    # on CUDA with SAE TP 1 and one hook.
    streaming_transport: Literal["auto", "device", "host"] = "auto"
    streaming_buffer_dir: str = "/dev/shm"
    # Transport of shard routing (`use_shard_routing`): "p2p" = row-router kernel over NVLink,
    # "collective" = torch.distributed point-to-point sends; "auto" = p2p on NCCL.
    routing_transport: Literal["auto", "p2p", "collective"] = "auto"

    # B200 engine knobs (no counterpart in the reference): use the fused native TopK-family
    # training step on CUDA when available ("auto"), always ("native") or never ("torch").
    sae_engine: Literal["auto", "native", "torch"] = "auto"
    # Tensor-parallel exchanges of the native engine: NVLink peer-memory kernels fused with the
    # compute ("p2p") or NCCL collectives between kernels ("nccl").
    tp_exchange: Literal["p2p", "nccl"] = "p2p"
    # Gradient all-reduce of `sae_dp_mode="ddp"` on the PyTorch path (SAEs without a native
    # engine): DDP's own NCCL all-reduce ("nccl", default: measured faster on the dense
    # JumpReLU step, where the all-reduce overlaps cuBLAS GEMMs) or a DDP communication hook
    # running the P2P all-reduce kernel ("p2p").  TopK-family SAEs use the native DDP engine.
    ddp_exchange: Literal["p2p", "nccl"] = "nccl"

    def __post_init__(self) -> None:
        if self.multi_sae_seed_mode not in ("same", "offset"):
            raise ValueError("multi_sae_seed_mode must be 'same' or 'offset'")
        if self.multi_sae_backward_order not in ("forward", "reverse", "largest_first"):
            raise ValueError("multi_sae_backward_order must be 'forward', 'reverse', or 'largest_first'")
        if self.multi_sae_stats_sync_mode not in ("immediate", "deferred", "periodic"):
            raise ValueError("multi_sae_stats_sync_mode must be 'immediate', 'deferred', or 'periodic'")
        if self.multi_sae_stats_sync_interval < 1:
            raise ValueError("multi_sae_stats_sync_interval must be >= 1")
        if self.ddp_bucket_cap_mb is not None and self.ddp_bucket_cap_mb <= 0:
            raise ValueError("ddp_bucket_cap_mb must be > 0 when set")
        if self.streaming_mode:
            if self.streaming_prefetch_chunks < 1:
                raise ValueError("streaming_prefetch_chunks must be >= 1.")
            if self.streaming_num_chunks <= self.streaming_prefetch_chunks:
                raise ValueError("streaming_num_chunks must be > streaming_prefetch_chunks.")
        if self.hook_names is not None:
            self.hook_names = list(dict.fromkeys(self.hook_names))
            if not self.hook_names:
                raise ValueError("hook_names must not be empty when provided")
            if len(self.hook_names) > 1 and self.sae_dp_mode == "manual":
                warnings.warn(
                    "Multi-layer SAE training does not use manual DP sync; defaulting sae_dp_mode to 'ddp'.",
                    stacklevel=2,
                )
                self.sae_dp_mode = "ddp"
            if len(self.hook_names) == 1:
                self.hook_name = self.hook_names[0]
        if self.sae_dp_mode == "ddp" and self.compile_sae:
            raise ValueError("compile_sae=True is incompatible with sae_dp_mode='ddp'.")
        if self.hook_eval != "NOT_IN_USE":
            warnings.warn("The 'hook_eval' field is deprecated and will be removed in v7.0.0. It is not used.",
                          DeprecationWarning, stacklevel=2)
        if self.use_cached_activations and self.cached_activations_path is None:
            if self.hook_names is not None and len(self.hook_names) > 1:
                raise ValueError("use_cached_activations is not supported with multi-layer hook_names.")
            self.cached_activations_path = _default_cached_activations_path(
                self.dataset_path, self.model_name, self.hook_name, self.hook_head_index)
        self.tokens_per_buffer = self.train_batch_size_tokens * self.context_size * self.n_batches_in_buffer
        if self.logger.run_name is None:
            self.logger.run_name = (
                f"{self.sae.architecture()}-{self.sae.d_sae}-LR-{self.lr}-Tokens-{self.training_tokens:3.3e}"
            )
        if self.model_from_pretrained_kwargs is None:
            self.model_from_pretrained_kwargs = (
                {"center_writing_weights": False} if self.model_class_name == "HookedTransformer" else {}
            )
        if self.act_store_device == "with_model":
            self.act_store_device = self.device
        if self.lr_end is None:
            self.lr_end = self.lr / 10
        for name in ("save_mse_every_n_steps", "save_timing_every_n_steps", "save_memory_every_n_steps"):
            v = getattr(self, name)
            if v < 0:
                raise ValueError(f"{name} must be >= 0")
            if v > 0 and self.output_path is None:
                raise ValueError(f"{name} requires output_path to be set")
        uid = self.logger.wandb_id
        if uid is None:
            uid = _timestamp_run_id()
            if self.checkpoint_path is not None:
                uid = _unique_run_id(Path(self.checkpoint_path), uid)
        if self.checkpoint_path is not None:
            self.checkpoint_path = str(Path(self.checkpoint_path) / uid)
        if self.verbose:
            steps = self.training_tokens // self.train_batch_size_tokens
            logger.info("Run name: %s; total training steps: %d", self.logger.run_name, steps)
        if self.context_size < 0:
            raise ValueError(f"The provided context_size is {self.context_size} is negative.")
        _validate_seqpos(self.seqpos_slice, self.context_size)
        if isinstance(self.exclude_special_tokens, list) and not all(
            isinstance(x, int) for x in self.exclude_special_tokens
        ):
            raise ValueError("exclude_special_tokens list must contain only integers")

    @property
    def total_training_tokens(self) -> int:
        return self.training_tokens

    @property
    def total_training_steps(self) -> int:
        return self.total_training_tokens // self.train_batch_size_tokens

    def get_training_sae_cfg_dict(self) -> dict[str, Any]:
        return self.sae.to_dict()

    def to_dict(self) -> dict[str, Any]:
        d = asdict(self)
        d["logger"] = asdict(self.logger)
        d["sae"] = self.sae.to_dict()
        d["dtype"] = str(self.dtype)
        d["device"] = str(self.device)
        d["act_store_device"] = str(self.act_store_device)
        return d

    @classmethod
    def from_dict(cls, cfg_dict: dict[str, Any]) -> LanguageModelSAERunnerConfig[Any]:
        if "sae" not in cfg_dict:
            raise ValueError("sae field is required in the config dictionary")
        if "architecture" not in cfg_dict["sae"]:
            raise ValueError("architecture field is required in the sae dictionary")
        if "logger" not in cfg_dict:
            raise ValueError("logger field is required in the config dictionary")
        sae_cfg = get_sae_training_class(cfg_dict["sae"]["architecture"])[1].from_dict(cfg_dict["sae"])
        d = {**cfg_dict, "sae": sae_cfg, "logger": LoggingConfig(**cfg_dict["logger"])}
        if isinstance(d.get("seqpos_slice"), list):
            d["seqpos_slice"] = tuple(d["seqpos_slice"])
        out = cls(**d)
        if "checkpoint_path" in cfg_dict:
            out.checkpoint_path = cfg_dict["checkpoint_path"]
        return out

    def to_sae_trainer_config(self) -> SAETrainerConfig:
        return SAETrainerConfig(
            n_checkpoints=self.n_checkpoints, checkpoint_path=self.checkpoint_path,
            save_final_checkpoint=self.save_final_checkpoint, output_path=self.output_path,
            save_mse_every_n_steps=self.save_mse_every_n_steps,
            save_timing_every_n_steps=self.save_timing_every_n_steps,
            save_memory_every_n_steps=self.save_memory_every_n_steps,
            synchronize_timing=self.synchronize_timing,
            multi_sae_backward_order=self.multi_sae_backward_order,
            multi_sae_stats_sync_mode=self.multi_sae_stats_sync_mode,
            multi_sae_stats_sync_interval=self.multi_sae_stats_sync_interval,
            total_training_samples=self.total_training_tokens, device=self.device, autocast=self.autocast,
            lr=self.lr, lr_end=self.lr_end, lr_scheduler_name=self.lr_scheduler_name,
            lr_warm_up_steps=self.lr_warm_up_steps, adam_beta1=self.adam_beta1, adam_beta2=self.adam_beta2,
            lr_decay_steps=self.lr_decay_steps, n_restart_cycles=self.n_restart_cycles,
            train_batch_size_samples=self.train_batch_size_tokens,
            dead_feature_window=self.dead_feature_window, feature_sampling_window=self.feature_sampling_window,
            logger=self.logger, sae_engine=self.sae_engine, tp_exchange=self.tp_exchange,
        )


@dataclass
class CacheActivationsRunnerConfig:
    """Configuration for caching LM activations to disk (sae_lens/config.py:597-765)."""

    dataset_path: str
    model_name: str
    model_batch_size: int
    hook_name: str
    d_in: int
    training_tokens: int
    context_size: int = -1
    model_class_name: str = "HookedTransformer"
    new_cached_activations_path: str | None = None
    shuffle: bool = True
    seed: int = 42
    dtype: str = "float32"
    device: str = field(default_factory=lambda: "cuda" if torch.cuda.is_available() else "cpu")
    buffer_size_gb: float = 2.0
    hf_repo_id: str | None = None
    hf_num_shards: int | None = None
    hf_revision: str = "main"
    hf_is_private_repo: bool = False
    model_kwargs: dict[str, Any] = field(default_factory=dict)
    model_from_pretrained_kwargs: dict[str, Any] = field(default_factory=dict)
    compile_llm: bool = False
    llm_compilation_mode: str | None = None
    prepend_bos: bool = True
    seqpos_slice: tuple[int | None, ...] = (None,)
    streaming: bool = True
    autocast_lm: bool = False
    dataset_trust_remote_code: bool | None = None

    def __post_init__(self) -> None:
        if self.context_size == -1:
            from saelens_b200.training.datasets import first_tokenized_length

            n = first_tokenized_length(self.dataset_path)
            if n is None:
                raise ValueError("Dataset is not tokenized. Please specify context_size.")
            self.context_size = n
        if self.seqpos_slice is not None:
            _validate_seqpos(self.seqpos_slice, self.context_size)
        if self.context_size > self.training_tokens:
            raise ValueError(
                f"context_size ({self.context_size}) is greater than training_tokens ({self.training_tokens})."
            )
        if self.new_cached_activations_path is None:
            self.new_cached_activations_path = _default_cached_activations_path(
                self.dataset_path, self.model_name, self.hook_name, None)

    @property
    def sliced_context_size(self) -> int:
        if self.seqpos_slice is not None:
            return len(range(self.context_size)[slice(*self.seqpos_slice)])
        return self.context_size

    @property
    def bytes_per_token(self) -> int:
        return self.d_in * str_to_dtype(self.dtype).itemsize

    @property
    def n_tokens_in_batch(self) -> int:
        return self.model_batch_size * self.sliced_context_size

    @property
    def n_tokens_in_buffer(self) -> int:
        t = int(self.buffer_size_gb * 1e9) // self.bytes_per_token
        return t - (t % self.n_tokens_in_batch)

    @property
    def n_batches_in_buffer(self) -> int:
        return self.n_tokens_in_buffer // self.n_tokens_in_batch

    @property
    def n_seq_in_dataset(self) -> int:
        return self.training_tokens // self.sliced_context_size

    @property
    def n_seq_in_buffer(self) -> int:
        return self.n_tokens_in_buffer // self.sliced_context_size

    @property
    def n_buffers(self) -> int:
        return math.ceil(self.training_tokens / self.n_tokens_in_buffer)


@dataclass
class PretokenizeRunnerConfig:
    tokenizer_name: str = "gpt2"
    dataset_path: str = ""
    dataset_name: str | None = None
    dataset_trust_remote_code: bool | None = None
    split: str | None = "train"
    data_files: list[str] | None = None
    data_dir: str | None = None
    num_proc: int = 4
    context_size: int = 128
    column_name: str = "text"
    shuffle: bool = True
    seed: int | None = None
    streaming: bool = False
    pretokenize_batch_size: int | None = 1000
    begin_batch_token: SpecialToken = "bos"
    begin_sequence_token: SpecialToken = None
    sequence_separator_token: SpecialToken = "bos"
    disable_concat_sequences: bool = False
    save_path: str | None = None
    hf_repo_id: str | None = None
    hf_num_shards: int = 64
    hf_revision: str = "main"
    hf_is_private_repo: bool = False


@dataclass
class SAETrainerConfig:
    n_checkpoints: int
    checkpoint_path: str | None
    save_final_checkpoint: bool
    output_path: str | None
    save_mse_every_n_steps: int
    save_timing_every_n_steps: int
    save_memory_every_n_steps: int
    synchronize_timing: bool
    multi_sae_backward_order: Literal["forward", "reverse", "largest_first"]
    multi_sae_stats_sync_mode: Literal["immediate", "deferred", "periodic"]
    multi_sae_stats_sync_interval: int
    total_training_samples: int
    device: str
    autocast: bool
    lr: float
    lr_end: float | None
    lr_scheduler_name: str
    lr_warm_up_steps: int
    adam_beta1: float
    adam_beta2: float
    lr_decay_steps: int
    n_restart_cycles: int
    train_batch_size_samples: int
    dead_feature_window: int
    feature_sampling_window: int
    logger: LoggingConfig
    sae_engine: Literal["auto", "native", "torch"] = "auto"
    tp_exchange: Literal["p2p", "nccl"] = "p2p"

    @property
    def total_training_steps(self) -> int:
        return self.total_training_samples // self.train_batch_size_samples
