"""SAE base classes: configs, metadata, inference `SAE` and `TrainingSAE`.

Public API and checkpoint layout follow the reference (sae_lens/saes/sae.py): weights
`W_enc [d_in, d_sae]`, `W_dec [d_sae, d_in]`, `b_enc [d_sae]`, `b_dec [d_in]` (plus
architecture-specific tensors) in `sae_weights.safetensors`, the config in `cfg.json`.
The PyTorch code here is the portable path (CPU and the oracle for the native kernels); the
fused sm_100a training step lives in `saelens_b200.training.engine`.
"""

from __future__ import annotations

import copy
import json
import warnings
from abc import ABC, abstractmethod
from collections.abc import Callable, Iterator
from contextlib import contextmanager
from dataclasses import asdict, dataclass, field, fields, replace
from pathlib import Path
from typing import TYPE_CHECKING, Any, Generic, Literal, NamedTuple, TypeVar

import torch
from safetensors.torch import load_file, save_file
from torch import nn

from saelens_b200 import __version__
from saelens_b200.constants import CHECKPOINT_FORMAT_VERSION, SAE_CFG_FILENAME, SAE_WEIGHTS_FILENAME
from saelens_b200.registry import get_sae_class, get_sae_training_class
from saelens_b200.utils.hooks import HookedRootModule, HookPoint
from saelens_b200.utils.misc import dtype_to_str, filter_valid_dataclass_fields, str_to_dtype

if TYPE_CHECKING:
    from saelens_b200.config import LanguageModelSAERunnerConfig

T_SAE_CONFIG = TypeVar("T_SAE_CONFIG", bound="SAEConfig")
T_TRAINING_SAE_CONFIG = TypeVar("T_TRAINING_SAE_CONFIG", bound="TrainingSAEConfig")
T_SAE = TypeVar("T_SAE", bound="SAE[Any]")
T_TRAINING_SAE = TypeVar("T_TRAINING_SAE", bound="TrainingSAE[Any]")


class SAEMetadata:
    """Free-form metadata (model name, hook name, ...); missing keys read as None."""

    def __init__(self, **kwargs: Any):
        self.sae_lens_version = kwargs.pop("sae_lens_version", CHECKPOINT_FORMAT_VERSION)
        self.sae_lens_training_version = kwargs.pop("sae_lens_training_version", CHECKPOINT_FORMAT_VERSION)
        self.saelens_b200_version = kwargs.pop("saelens_b200_version", __version__)
        for k, v in kwargs.items():
            setattr(self, k, v)

    def __getattr__(self, name: str) -> Any:
        if name.startswith("__"):
            raise AttributeError(name)
        return None

    def __getitem__(self, key: str) -> Any:
        return getattr(self, key)

    def __setitem__(self, key: str, value: Any) -> None:
        setattr(self, key, value)

    def __contains__(self, key: str) -> bool:
        return key in self.__dict__

    def get(self, key: str, default: Any = None) -> Any:
        return self.__dict__.get(key, default)

    def keys(self):
        return self.__dict__.keys()

    def values(self):
        return self.__dict__.values()

    def items(self):
        return self.__dict__.items()

    def to_dict(self) -> dict[str, Any]:
        return dict(self.__dict__)

    @classmethod
    def from_dict(cls, data: dict[str, Any]) -> SAEMetadata:
        return cls(**data)

    def __repr__(self) -> str:
        return f"SAEMetadata({self.__dict__})"

    def __eq__(self, other: object) -> bool:
        return isinstance(other, SAEMetadata) and self.__dict__ == other.__dict__

    def __deepcopy__(self, memo: dict[int, Any]) -> SAEMetadata:
        return SAEMetadata(**copy.deepcopy(self.__dict__, memo))

    def __getstate__(self) -> dict[str, Any]:
        return self.__dict__

    def __setstate__(self, state: dict[str, Any]) -> None:
        self.__dict__.update(state)


NormalizeMode = Literal["none", "expected_average_only_in", "constant_norm_rescale", "layer_norm"]


@dataclass
class SAEConfig(ABC):
    d_in: int
    d_sae: int
    dtype: str = "float32"
    device: str = "cpu"
    apply_b_dec_to_input: bool = True
    normalize_activations: NormalizeMode = "none"
    reshape_activations: Literal["none", "hook_z"] = "none"
    metadata: SAEMetadata = field(default_factory=SAEMetadata)

    @classmethod
    @abstractmethod
    def architecture(cls) -> str: ...

    def __post_init__(self) -> None:
        if self.normalize_activations not in (
            "none", "expected_average_only_in", "constant_norm_rescale", "layer_norm",
        ):
            raise ValueError(
                "normalize_activations must be none, expected_average_only_in, layer_norm, or "
                f"constant_norm_rescale. Got {self.normalize_activations}"
            )

    def to_dict(self) -> dict[str, Any]:
        d = {f.name: getattr(self, f.name) for f in fields(self)}
        d["metadata"] = self.metadata.to_dict()
        d["architecture"] = self.architecture()
        return d

    @classmethod
    def from_dict(cls: type[T_SAE_CONFIG], config_dict: dict[str, Any]) -> T_SAE_CONFIG:
        cfg_class = get_sae_class(config_dict["architecture"])[1]
        res = cfg_class(**filter_valid_dataclass_fields(config_dict, cfg_class))
        if "metadata" in config_dict:
            res.metadata = SAEMetadata(**config_dict["metadata"])
        if not isinstance(res, cls):
            raise ValueError(f"SAE config class {cls} does not match dict config class {type(res)}")
        return res


@dataclass
class TrainStepOutput:
    sae_in: torch.Tensor
    sae_out: torch.Tensor
    feature_acts: torch.Tensor
    hidden_pre: torch.Tensor
    loss: torch.Tensor
    losses: dict[str, torch.Tensor]
    metrics: dict[str, Any] = field(default_factory=dict)


@dataclass
class TrainStepInput:
    sae_in: torch.Tensor
    coefficients: dict[str, float]
    dead_neuron_mask: torch.Tensor | None
    n_training_steps: int = 0
    is_logging_step: bool = False


class TrainCoefficientConfig(NamedTuple):
    value: float
    warm_up_steps: int


_blank = nn.Identity()


@contextmanager
def _disable_hooks(sae: SAE[Any]) -> Iterator[None]:
    saved = dict(sae.hook_dict)
    try:
        for name in saved:
            setattr(sae, name, _blank)
        yield
    finally:
        for name, hp in saved.items():
            setattr(sae, name, hp)


class SAE(HookedRootModule, Generic[T_SAE_CONFIG], ABC):
    """Inference SAE.  Subclasses implement `encode` / `decode` (+ weight init)."""

    cfg: T_SAE_CONFIG
    W_enc: nn.Parameter
    W_dec: nn.Parameter
    b_dec: nn.Parameter

    def __init__(self, cfg: T_SAE_CONFIG, use_error_term: bool = False):
        super().__init__()
        self.cfg = cfg
        if cfg.metadata and cfg.metadata.model_from_pretrained_kwargs:
            warnings.warn(
                "This SAE has non-empty model_from_pretrained_kwargs; load the model with them.",
                UserWarning, stacklevel=1,
            )
        self.dtype = str_to_dtype(cfg.dtype)
        self.device = torch.device(cfg.device)
        self._use_error_term = False
        if use_error_term:
            self.use_error_term = True
        self.activation_fn = self.get_activation_fn()
        self.initialize_weights()
        self.hook_sae_input = HookPoint()
        self.hook_sae_acts_pre = HookPoint()
        self.hook_sae_acts_post = HookPoint()
        self.hook_sae_output = HookPoint()
        self.hook_sae_recons = HookPoint()
        self.hook_sae_error = HookPoint()
        if cfg.reshape_activations == "hook_z":
            self.turn_on_forward_pass_hook_z_reshaping()
        else:
            self.turn_off_forward_pass_hook_z_reshaping()
        self._setup_activation_normalization()
        self.setup()

    # ------------------------------------------------------------------ properties
    @property
    def use_error_term(self) -> bool:
        return self._use_error_term

    @use_error_term.setter
    def use_error_term(self, value: bool) -> None:
        if value and not self._use_error_term:
            warnings.warn(
                "Setting use_error_term directly on SAE is deprecated; use "
                "HookedSAETransformer.add_sae(sae, use_error_term=True).",
                DeprecationWarning, stacklevel=2,
            )
        self._use_error_term = value

    # ------------------------------------------------------------------ init
    def get_activation_fn(self) -> Callable[[torch.Tensor], torch.Tensor]:
        return nn.ReLU()

    def initialize_weights(self) -> None:
        """Kaiming-uniform decoder, encoder tied to its transpose, zero b_dec."""
        self.b_dec = nn.Parameter(torch.zeros(self.cfg.d_in, dtype=self.dtype, device=self.device))
        w = torch.empty(self.cfg.d_sae, self.cfg.d_in, dtype=self.dtype, device=self.device)
        nn.init.kaiming_uniform_(w)
        self.W_dec = nn.Parameter(w)
        self.W_enc = nn.Parameter(w.T.contiguous())

    def _setup_activation_normalization(self) -> None:
        mode = self.cfg.normalize_activations
        if mode == "constant_norm_rescale":
            def fn_in(x: torch.Tensor) -> torch.Tensor:
                self.x_norm_coeff = (self.cfg.d_in ** 0.5) / x.norm(dim=-1, keepdim=True)
                return x * self.x_norm_coeff

            def fn_out(x: torch.Tensor) -> torch.Tensor:
                x = x / self.x_norm_coeff
                del self.x_norm_coeff
                return x

        elif mode == "layer_norm":
            def fn_in(x: torch.Tensor, eps: float = 1e-5) -> torch.Tensor:
                mu = x.mean(dim=-1, keepdim=True)
                x = x - mu
                std = x.std(dim=-1, keepdim=True)
                self.ln_mu, self.ln_std = mu, std
                return x / (std + eps)

            def fn_out(x: torch.Tensor, eps: float = 1e-5) -> torch.Tensor:  # noqa: ARG001
                return x * self.ln_std + self.ln_mu

        else:
            def fn_in(x: torch.Tensor) -> torch.Tensor:
                return x

            def fn_out(x: torch.Tensor) -> torch.Tensor:
                return x

        self.run_time_activation_norm_fn_in = fn_in
        self.run_time_activation_norm_fn_out = fn_out

    def turn_on_forward_pass_hook_z_reshaping(self) -> None:
        hook_name = self.cfg.metadata.hook_name
        if hook_name is not None and not hook_name.endswith("_z"):
            raise ValueError("This method should only be called for hook_z SAEs.")

        def reshape_in(x: torch.Tensor) -> torch.Tensor:
            self.d_head = x.shape[-1]
            return x.reshape(*x.shape[:-2], x.shape[-2] * x.shape[-1])

        self.reshape_fn_in = reshape_in
        self.reshape_fn_out = lambda x, d_head: x.reshape(*x.shape[:-1], x.shape[-1] // d_head, d_head)
        self.hook_z_reshaping_mode = True

    def turn_off_forward_pass_hook_z_reshaping(self) -> None:
        self.reshape_fn_in = lambda x: x
        self.reshape_fn_out = lambda x, d_head: x  # noqa: ARG005
        self.d_head = None
        self.hook_z_reshaping_mode = False

    # ------------------------------------------------------------------ device / dtype
    def to(self: T_SAE, *args: Any, **kwargs: Any) -> T_SAE:  # type: ignore[override]
        device_arg = kwargs.get("device")
        dtype_arg = kwargs.get("dtype")
        for a in args:
            if isinstance(a, (torch.device, str)):
                device_arg = a
            elif isinstance(a, torch.dtype):
                dtype_arg = a
            elif isinstance(a, torch.Tensor):
                device_arg, dtype_arg = a.device, a.dtype
        if device_arg is not None:
            dev = torch.device(device_arg) if isinstance(device_arg, str) else device_arg
            self.cfg.device = str(dev)
            self.device = dev
        if dtype_arg is not None:
            self.cfg.dtype = dtype_to_str(dtype_arg)
            self.dtype = dtype_arg
        return super().to(*args, **kwargs)

    # ------------------------------------------------------------------ forward
    @abstractmethod
    def encode(self, x: torch.Tensor) -> torch.Tensor: ...

    @abstractmethod
    def decode(self, feature_acts: torch.Tensor) -> torch.Tensor: ...

    def process_sae_in(self, sae_in: torch.Tensor) -> torch.Tensor:
        sae_in = sae_in.to(self.dtype)
        sae_in = self.reshape_fn_in(sae_in)
        sae_in = self.hook_sae_input(sae_in)
        sae_in = self.run_time_activation_norm_fn_in(sae_in)
        return sae_in - self.b_dec * self.cfg.apply_b_dec_to_input

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        feature_acts = self.encode(x)
        sae_out = self.decode(feature_acts)
        if self.use_error_term:
            with torch.no_grad(), _disable_hooks(self):
                clean = self.decode(self.encode(x))
            sae_error = self.hook_sae_error(x - clean)
            sae_out = sae_out + sae_error
        return self.hook_sae_output(sae_out)

    # ------------------------------------------------------------------ hooks for subclasses
    def process_state_dict_for_saving(self, state_dict: dict[str, Any]) -> None:
        pass

    def process_state_dict_for_loading(self, state_dict: dict[str, Any]) -> None:
        pass

    def process_named_optimizer_state_for_saving(self, optimizer_state: dict[str, dict[str, Any]]) -> None:
        pass

    def process_named_optimizer_state_for_loading(self, optimizer_state: dict[str, dict[str, Any]]) -> None:
        pass

    def sync_tensor_parallel_gradients(self) -> None:
        pass

    def clip_grad_norm_(self, max_norm: float, dp_group: Any = None) -> torch.Tensor:  # noqa: ARG002
        return torch.nn.utils.clip_grad_norm_(self.parameters(), max_norm)

    # ------------------------------------------------------------------ weight utilities
    @torch.no_grad()
    def fold_activation_norm_scaling_factor(self, scaling_factor: float) -> None:
        self.W_enc.data *= scaling_factor
        self.W_dec.data /= scaling_factor
        self.b_dec.data /= scaling_factor
        self.cfg.normalize_activations = "none"

    @torch.no_grad()
    def fold_W_dec_norm(self) -> None:
        norms = self.W_dec.norm(dim=-1).clamp(min=1e-8).unsqueeze(1)
        self.W_dec.data = self.W_dec.data / norms
        self.W_enc.data = self.W_enc.data * norms.T
        if isinstance(getattr(self, "b_enc", None), nn.Parameter):
            self.b_enc.data = self.b_enc.data * norms.squeeze()

    def get_name(self) -> str:
        return f"sae_{self.cfg.metadata.model_name}_{self.cfg.metadata.hook_name}_{self.cfg.d_sae}"

    # ------------------------------------------------------------------ save / load
    def save_model(self, path: str | Path) -> tuple[Path, Path]:
        path = Path(path)
        path.mkdir(parents=True, exist_ok=True)
        sd = {k: v.contiguous() for k, v in self.state_dict().items()}
        self.process_state_dict_for_saving(sd)
        wpath = path / SAE_WEIGHTS_FILENAME
        save_file({k: v.contiguous() for k, v in sd.items()}, wpath)
        cpath = path / SAE_CFG_FILENAME
        with open(cpath, "w") as f:
            json.dump(self.cfg.to_dict(), f)
        return wpath, cpath

    @classmethod
    def get_sae_class_for_architecture(cls: type[T_SAE], architecture: str) -> type[T_SAE]:
        sae_cls, _ = get_sae_class(architecture)
        if not issubclass(sae_cls, cls):
            raise ValueError(f"Loaded SAE is not of type {cls.__name__}. Use {sae_cls.__name__} instead")
        return sae_cls

    @classmethod
    def get_sae_config_class_for_architecture(cls, architecture: str) -> type[SAEConfig]:  # noqa: ARG003
        return SAEConfig

    @classmethod
    def _build_from(cls: type[T_SAE], cfg_dict: dict[str, Any], state_dict: dict[str, torch.Tensor]) -> T_SAE:
        from saelens_b200.loading.pretrained_sae_loaders import handle_config_defaulting

        cfg_dict = handle_config_defaulting(cfg_dict)
        cfg_cls = cls.get_sae_config_class_for_architecture(cfg_dict["architecture"])
        cfg = cfg_cls.from_dict(cfg_dict)
        sae_cls = cls.get_sae_class_for_architecture(cfg.architecture())
        device = cfg.device
        cfg.device = "meta"
        sae = sae_cls(cfg)
        sae.cfg.device = device
        sae.process_state_dict_for_loading(state_dict)
        sae.load_state_dict(state_dict, assign=True)
        return sae.to(dtype=str_to_dtype(cfg.dtype), device=device)

    @classmethod
    def load_from_disk(cls: type[T_SAE], path: str | Path, device: str = "cpu",
                       dtype: str | None = None, converter: Any = None) -> T_SAE:
        from saelens_b200.loading.pretrained_sae_loaders import sae_lens_disk_loader

        overrides = {"dtype": dtype} if dtype is not None else None
        conv = converter or sae_lens_disk_loader
        cfg_dict, state_dict = conv(path, device, cfg_overrides=overrides)
        return cls._build_from(cfg_dict, state_dict)

    @classmethod
    def load_from_pretrained(cls: type[T_SAE], path: str | Path, device: str = "cpu",
                             dtype: str | None = None) -> T_SAE:
        return cls.load_from_disk(path, device=device, dtype=dtype)

    @classmethod
    def from_pretrained(cls: type[T_SAE], release: str, sae_id: str, device: str = "cpu",
                        dtype: str = "float32", force_download: bool = False,
                        converter: Any = None) -> T_SAE:
        return cls.from_pretrained_with_cfg_and_sparsity(
            release, sae_id, device, dtype=dtype, force_download=force_download, converter=converter,
        )[0]

    @classmethod
    def from_pretrained_with_cfg_and_sparsity(
        cls: type[T_SAE], release: str, sae_id: str, device: str = "cpu", dtype: str = "float32",
        force_download: bool = False, converter: Any = None,
    ) -> tuple[T_SAE, dict[str, Any], torch.Tensor | None]:
        from saelens_b200.loading.pretrained_sae_loaders import (
            NAMED_PRETRAINED_SAE_LOADERS,
            handle_config_defaulting,
        )
        from saelens_b200.loading.pretrained_saes_directory import (
            get_config_overrides,
            get_conversion_loader_name,
            get_norm_scaling_factor,
            get_pretrained_saes_directory,
            get_repo_id_and_folder_name,
        )

        directory = get_pretrained_saes_directory()
        if release not in directory and "/" not in release:
            raise ValueError(
                f"Release {release} not found in pretrained SAEs directory, and is not a valid "
                "huggingface repo."
            )
        if release in directory and sae_id not in directory[release].saes_map:
            ids = list(directory[release].saes_map)
            raise ValueError(f"ID {sae_id} not found in release {release}. Valid IDs are {ids[:5]}.")
        loader = converter or NAMED_PRETRAINED_SAE_LOADERS[get_conversion_loader_name(release)]
        repo_id, folder = get_repo_id_and_folder_name(release, sae_id)
        overrides = get_config_overrides(release, sae_id)
        overrides["device"] = device
        overrides["dtype"] = dtype
        cfg_dict, state_dict, log_sparsity = loader(
            repo_id=repo_id, folder_name=folder, device=device, force_download=force_download,
            cfg_overrides=overrides,
        )
        cfg_dict = handle_config_defaulting(cfg_dict)
        sae = cls._build_from(cfg_dict, state_dict)
        if cfg_dict.get("normalize_activations") == "expected_average_only_in":
            factor = get_norm_scaling_factor(release, sae_id)
            if factor is not None:
                sae.fold_activation_norm_scaling_factor(factor)
                cfg_dict["normalize_activations"] = "none"
            else:
                warnings.warn(
                    f"norm_scaling_factor not found for {release} and {sae_id}; skipping folding.",
                    stacklevel=2,
                )
        return sae.to(dtype=str_to_dtype(dtype), device=device), cfg_dict, log_sparsity

    @classmethod
    def from_dict(cls: type[T_SAE], config_dict: dict[str, Any]) -> T_SAE:
        sae_cls = cls.get_sae_class_for_architecture(config_dict["architecture"])
        cfg_cls = cls.get_sae_config_class_for_architecture(config_dict["architecture"])
        return sae_cls(cfg_cls.from_dict(config_dict))

    # deprecated tuple-like access (from_pretrained used to return a tuple)
    def __getitem__(self, index: int) -> Any:
        warnings.warn("Indexing SAE objects is deprecated.", DeprecationWarning, stacklevel=2)
        return (self, self.cfg.to_dict(), None)[index]

    def __iter__(self):
        warnings.warn("Unpacking SAE objects is deprecated.", DeprecationWarning, stacklevel=2)
        return iter((self, self.cfg.to_dict(), None))

    def __len__(self) -> int:
        warnings.warn("Getting length of SAE objects is deprecated.", DeprecationWarning, stacklevel=2)
        return 3


@dataclass(kw_only=True)
class TrainingSAEConfig(SAEConfig, ABC):
    decoder_init_norm: float | None = 0.1

    @classmethod
    @abstractmethod
    def architecture(cls) -> str: ...

    @classmethod
    def from_sae_runner_config(cls: type[T_TRAINING_SAE_CONFIG],
                               cfg: LanguageModelSAERunnerConfig[T_TRAINING_SAE_CONFIG]) -> T_TRAINING_SAE_CONFIG:
        metadata = SAEMetadata(
            model_name=cfg.model_name,
            hook_name=cfg.hook_name,
            hook_head_index=cfg.hook_head_index,
            context_size=cfg.context_size,
            prepend_bos=cfg.prepend_bos,
            seqpos_slice=cfg.seqpos_slice,
            model_from_pretrained_kwargs=cfg.model_from_pretrained_kwargs or {},
        )
        if not isinstance(cfg.sae, cls):
            raise ValueError(f"SAE config class {cls} does not match SAE runner config class {type(cfg.sae)}")
        return replace(cfg.sae, metadata=metadata)

    @classmethod
    def from_dict(cls: type[T_TRAINING_SAE_CONFIG], config_dict: dict[str, Any]) -> T_TRAINING_SAE_CONFIG:
        cfg_class: type[Any] = cls
        if "architecture" in config_dict:
            cfg_class = get_sae_training_class(config_dict["architecture"])[1]
        if not issubclass(cfg_class, cls):
            raise ValueError(f"SAE config class {cls} does not match dict config class {cfg_class}")
        valid = filter_valid_dataclass_fields(config_dict, cfg_class)
        if "metadata" in config_dict:
            valid["metadata"] = SAEMetadata(**config_dict["metadata"])
        return cfg_class(**valid)

    def to_dict(self) -> dict[str, Any]:
        d = asdict(self)
        d["metadata"] = self.metadata.to_dict()
        d["architecture"] = self.architecture()
        return d

    def get_inference_config_class(self) -> type[SAEConfig]:
        return get_sae_class(self.architecture())[1]

    def get_inference_sae_cfg_dict(self) -> dict[str, Any]:
        base = self.get_inference_config_class()
        names = {f.name for f in fields(base)}
        d = {n: getattr(self, n) for n in names}
        d["architecture"] = base.architecture()
        d["metadata"] = self.metadata.to_dict()
        return d


class TrainingSAE(SAE[T_TRAINING_SAE_CONFIG], ABC):
    """Training SAE: adds `training_forward_pass` (MSE + architecture losses)."""

    def __init__(self, cfg: T_TRAINING_SAE_CONFIG, use_error_term: bool = False):
        super().__init__(cfg, use_error_term)
        self.turn_off_forward_pass_hook_z_reshaping()
        self.mse_loss_fn = mse_loss

    def forward(self, x: torch.Tensor | TrainStepInput) -> Any:  # type: ignore[override]
        if isinstance(x, TrainStepInput):
            return self.training_forward_pass(x)
        return super().forward(x)

    @abstractmethod
    def get_coefficients(self) -> dict[str, float | TrainCoefficientConfig]: ...

    @abstractmethod
    def encode_with_hidden_pre(self, x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]: ...

    @abstractmethod
    def calculate_aux_loss(self, step_input: TrainStepInput, feature_acts: torch.Tensor,
                           hidden_pre: torch.Tensor, sae_out: torch.Tensor) -> Any: ...

    def encode(self, x: torch.Tensor) -> torch.Tensor:
        return self.encode_with_hidden_pre(x)[0]

    def decode(self, feature_acts: torch.Tensor) -> torch.Tensor:
        out = feature_acts @ self.W_dec + self.b_dec
        out = self.hook_sae_recons(out)
        out = self.run_time_activation_norm_fn_out(out)
        return self.reshape_fn_out(out, self.d_head)

    def initialize_weights(self) -> None:
        super().initialize_weights()
        if self.cfg.decoder_init_norm is not None:
            with torch.no_grad():
                self.W_dec.data /= self.W_dec.norm(dim=-1, keepdim=True)
                self.W_dec.data *= self.cfg.decoder_init_norm
            self.W_enc.data = self.W_dec.data.T.contiguous()

    def training_forward_pass(self, step_input: TrainStepInput) -> TrainStepOutput:
        feature_acts, hidden_pre = self.encode_with_hidden_pre(step_input.sae_in)
        sae_out = self.decode(feature_acts)
        mse = self.mse_loss_fn(sae_out, step_input.sae_in).sum(dim=-1).mean()
        aux = self.calculate_aux_loss(step_input=step_input, feature_acts=feature_acts,
                                      hidden_pre=hidden_pre, sae_out=sae_out)
        losses: dict[str, torch.Tensor] = {"mse_loss": mse}
        total = mse
        if isinstance(aux, dict):
            losses.update(aux)
            for v in aux.values():
                total = total + v
        else:
            total = total + aux
        return TrainStepOutput(sae_in=step_input.sae_in, sae_out=sae_out, feature_acts=feature_acts,
                               hidden_pre=hidden_pre, loss=total, losses=losses)

    def save_inference_model(self, path: str | Path) -> tuple[Path, Path]:
        path = Path(path)
        path.mkdir(parents=True, exist_ok=True)
        sd = {k: v.contiguous() for k, v in self.state_dict().items()}
        self.process_state_dict_for_saving_inference(sd)
        wpath = path / SAE_WEIGHTS_FILENAME
        save_file({k: v.contiguous() for k, v in sd.items()}, wpath)
        cpath = path / SAE_CFG_FILENAME
        with open(cpath, "w") as f:
            json.dump(self.cfg.get_inference_sae_cfg_dict(), f)
        return wpath, cpath

    def process_state_dict_for_saving_inference(self, state_dict: dict[str, Any]) -> None:
        self.process_state_dict_for_saving(state_dict)

    @torch.no_grad()
    def log_histograms(self) -> dict[str, Any]:
        return {"weights/W_dec_norms": self.W_dec.detach().float().norm(dim=1).cpu().numpy()}

    @classmethod
    def get_sae_class_for_architecture(cls: type[T_TRAINING_SAE], architecture: str) -> type[T_TRAINING_SAE]:
        sae_cls, _ = get_sae_training_class(architecture)
        if not issubclass(sae_cls, cls):
            raise ValueError(f"Loaded SAE is not of type {cls.__name__}. Use {sae_cls.__name__} instead")
        return sae_cls

    @classmethod
    def get_sae_config_class_for_architecture(cls, architecture: str) -> type[TrainingSAEConfig]:
        return get_sae_training_class(architecture)[1]

    def load_weights_from_checkpoint(self, checkpoint_path: Path | str) -> None:
        sd = load_file(Path(checkpoint_path) / SAE_WEIGHTS_FILENAME)
        self.process_state_dict_for_loading(sd)
        self.load_state_dict(sd)


def mse_loss(preds: torch.Tensor, target: torch.Tensor) -> torch.Tensor:
    return torch.nn.functional.mse_loss(preds, target, reduction="none")
