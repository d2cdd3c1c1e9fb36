"""TopK SAEs, including latent-sharded tensor parallelism.

Semantics follow sae_lens/saes/topk_sae.py: per-row top-k of the (decoder-norm rescaled)
pre-activations, ReLU on the selected values, decode with the inverse rescale; the aux-k loss
makes the top d_in/2 dead latents reconstruct the residual (topk_sae.py:710-813).

Tensor parallelism (topk_sae.py:448-674): `shard_weights(group)` keeps W_enc[:, shard],
W_dec[shard], b_enc[shard]; b_dec stays replicated.  The forward all-gathers the local
pre-activations for the full-width top-k, decodes the local shard and all-reduces the partial
reconstruction.  Unlike the reference, the SAE input passes through `tp_copy`, so the gradient
reaching b_dec through the encoder sums over every shard and matches TP=1 exactly.

This module is the portable PyTorch path.  On CUDA the trainer runs TopK-family SAEs through
the fused native engine (`saelens_b200.training.engine`), which never materialises the dense
[batch, d_sae] activations.
"""

from __future__ import annotations

import json
from collections.abc import Callable
from dataclasses import dataclass
from pathlib import Path
from typing import Any

import torch
import torch.distributed as dist
from safetensors.torch import save_file
from torch import nn

from saelens_b200.constants import SAE_CFG_FILENAME, SAE_WEIGHTS_FILENAME
from saelens_b200.models.sae import (
    SAE,
    SAEConfig,
    TrainCoefficientConfig,
    TrainingSAE,
    TrainingSAEConfig,
    TrainStepInput,
)
from saelens_b200.parallel.profiling import nccl_nvtx_range
from saelens_b200.parallel.tp import tp_allgather, tp_allreduce, tp_copy
from saelens_b200.utils.hooks import HookPoint


class SparseHookPoint(HookPoint):
    """Hook point that densifies sparse inputs only when a hook is attached."""

    def __init__(self, d_sae: int):
        super().__init__()
        self.d_sae = d_sae

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if self.has_hooks and x.is_sparse:
            return x.to_dense()
        return x


class TopK(nn.Module):
    """Keep the k largest entries of the last dim, ReLU them, zero the rest."""

    def __init__(self, k: int, use_sparse_activations: bool = False):
        super().__init__()
        self.k = k
        self.use_sparse_activations = use_sparse_activations

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        vals, idx = torch.topk(x, k=self.k, dim=-1, sorted=False)
        vals = vals.relu()
        if self.use_sparse_activations:
            lead = x.shape[:-1]
            n_rows = int(torch.tensor(lead).prod().item()) if len(lead) else 1
            rows = torch.arange(n_rows, device=x.device).repeat_interleave(self.k)
            coords = [rows] if len(lead) == 1 else list(torch.unravel_index(rows, lead))
            ind = torch.stack([*coords, idx.flatten()])
            return torch.sparse_coo_tensor(ind, vals.flatten(), x.shape)
        return torch.zeros_like(x).scatter_(-1, idx, vals)


def _sparse_matmul(sparse: torch.Tensor, dense: torch.Tensor) -> torch.Tensor:
    """[..., d_sae] sparse COO times [d_sae, d_out] dense."""
    lead = sparse.shape[:-1]
    if sparse.ndim == 2:
        with torch.autocast(device_type=sparse.device.type, enabled=False):
            return torch.sparse.mm(sparse, dense)
    sp = sparse.coalesce()
    ind, val = sp.indices(), sp.values()
    flat = torch.zeros_like(ind[0])
    mul = 1
    for i in reversed(range(len(lead))):
        flat = flat + ind[i] * mul
        mul *= lead[i]
    n = int(torch.tensor(lead).prod().item())
    sp2 = torch.sparse_coo_tensor(torch.stack([flat, ind[-1]]), val, (n, sparse.shape[-1])).coalesce()
    with torch.autocast(device_type=sparse.device.type, enabled=False):
        out = torch.sparse.mm(sp2, dense)
    return out.view(*lead, dense.shape[-1])


def act_times_W_dec(feature_acts: torch.Tensor, W_dec: torch.Tensor,
                    rescale_acts_by_decoder_norm: bool) -> torch.Tensor:
    if rescale_acts_by_decoder_norm:
        feature_acts = feature_acts * (1 / W_dec.norm(dim=-1))
    if feature_acts.is_sparse:
        return _sparse_matmul(feature_acts, W_dec)
    return feature_acts @ W_dec


def _fold_norm_topk(W_enc: torch.Tensor, b_enc: torch.Tensor, W_dec: torch.Tensor) -> None:
    n = W_dec.norm(dim=-1).clamp(min=1e-8)
    b_enc.data = b_enc.data * n
    W_dec.data = W_dec.data / n.unsqueeze(1)
    W_enc.data = W_enc.data * n.unsqueeze(0)


@dataclass
class TopKSAEConfig(SAEConfig):
    k: int = 100
    rescale_acts_by_decoder_norm: bool = False

    @classmethod
    def architecture(cls) -> str:
        return "topk"


class TopKSAE(SAE[TopKSAEConfig]):
    b_enc: nn.Parameter

    def initialize_weights(self) -> None:
        super().initialize_weights()
        self.b_enc = nn.Parameter(torch.zeros(self.cfg.d_sae, dtype=self.dtype, device=self.device))

    def get_activation_fn(self) -> Callable[[torch.Tensor], torch.Tensor]:
        return TopK(self.cfg.k)

    def encode(self, x: torch.Tensor) -> torch.Tensor:
        sae_in = self.process_sae_in(x)
        pre = self.hook_sae_acts_pre(sae_in @ self.W_enc + self.b_enc)
        if self.cfg.rescale_acts_by_decoder_norm:
            pre = pre * self.W_dec.norm(dim=-1)
        return self.hook_sae_acts_post(self.activation_fn(pre))

    def decode(self, feature_acts: torch.Tensor) -> torch.Tensor:
        out = act_times_W_dec(feature_acts, self.W_dec, self.cfg.rescale_acts_by_decoder_norm) + self.b_dec
        out = self.hook_sae_recons(out)
        out = self.run_time_activation_norm_fn_out(out)
        return self.reshape_fn_out(out, self.d_head)

    @torch.no_grad()
    def fold_W_dec_norm(self) -> None:
        if not self.cfg.rescale_acts_by_decoder_norm:
            raise NotImplementedError(
                "Folding W_dec_norm is not safe for TopKSAEs when rescale_acts_by_decoder_norm is "
                "False, as this may change the topk activations"
            )
        _fold_norm_topk(self.W_enc, self.b_enc, self.W_dec)


@dataclass
class TopKTrainingSAEConfig(TrainingSAEConfig):
    k: int = 100
    use_sparse_activations: bool = False
    aux_loss_coefficient: float = 1.0
    rescale_acts_by_decoder_norm: bool = True

    @classmethod
    def architecture(cls) -> str:
        return "topk"


def calculate_topk_aux_acts(k_aux: int, hidden_pre: torch.Tensor,
                            dead_neuron_mask: torch.Tensor) -> torch.Tensor:
    """Activations of the top-k_aux dead latents (raw values, no ReLU), zeros elsewhere."""
    masked = torch.where(dead_neuron_mask[None], hidden_pre, -torch.inf)
    top = masked.topk(k_aux, sorted=False)
    return torch.zeros_like(hidden_pre).scatter_(-1, top.indices, top.values)


class TopKTrainingSAE(TrainingSAE[TopKTrainingSAEConfig]):
    b_enc: nn.Parameter

    def __init__(self, cfg: TopKTrainingSAEConfig, use_error_term: bool = False):
        super().__init__(cfg, use_error_term)
        self._tp_group: dist.ProcessGroup | None = None
        self.hook_sae_acts_post = SparseHookPoint(self.cfg.d_sae)
        self.setup()

    def initialize_weights(self) -> None:
        super().initialize_weights()
        self.b_enc = nn.Parameter(torch.zeros(self.cfg.d_sae, dtype=self.dtype, device=self.device))

    def get_activation_fn(self) -> Callable[[torch.Tensor], torch.Tensor]:
        return TopK(self.cfg.k, use_sparse_activations=self.cfg.use_sparse_activations)

    def get_coefficients(self) -> dict[str, float | TrainCoefficientConfig]:
        return {}

    # ---------------------------------------------------------------- tensor parallelism
    @staticmethod
    def _tp_param_shard_dims() -> dict[str, int | None]:
        return {"W_enc": 1, "W_dec": 0, "b_enc": 0, "b_dec": None}

    @property
    def tp_group(self) -> dist.ProcessGroup | None:
        return self._tp_group

    def _tp_info(self) -> tuple[int, int]:
        if self._tp_group is None:
            return 0, 1
        return dist.get_rank(self._tp_group), dist.get_world_size(self._tp_group)

    def shard_weights(self, tp_group: dist.ProcessGroup) -> None:
        rank, size = dist.get_rank(tp_group), dist.get_world_size(tp_group)
        if self.cfg.d_sae % size != 0:
            raise ValueError(f"d_sae={self.cfg.d_sae} must be divisible by tp_size={size}")
        n = self.cfg.d_sae // size
        s = rank * n
        self._tp_group = tp_group
        self.W_enc = nn.Parameter(self.W_enc.data[:, s : s + n].contiguous())
        self.W_dec = nn.Parameter(self.W_dec.data[s : s + n].contiguous())
        self.b_enc = nn.Parameter(self.b_enc.data[s : s + n].contiguous())

    def _gather_tp_tensor(self, t: torch.Tensor, dim: int | None) -> torch.Tensor:
        if self._tp_group is None or dim is None:
            return t.detach().clone()
        size = dist.get_world_size(self._tp_group)
        parts = [torch.empty_like(t) for _ in range(size)]
        with nccl_nvtx_range("nccl:topk_tp_state_all_gather", self._tp_group):
            dist.all_gather(parts, t.detach().contiguous(), group=self._tp_group)
        return torch.cat(parts, dim=dim)

    def _slice_tp_tensor(self, t: torch.Tensor, dim: int | None) -> torch.Tensor:
        if self._tp_group is None or dim is None:
            return t
        rank, size = self._tp_info()
        if t.shape[dim] % size != 0:
            raise ValueError(f"shape {tuple(t.shape)} dim {dim} not divisible by tp_size={size}")
        n = t.shape[dim] // size
        return t.narrow(dim, rank * n, n).contiguous()

    def process_state_dict_for_saving(self, state_dict: dict[str, Any]) -> None:
        if self._tp_group is None:
            return
        for name, dim in self._tp_param_shard_dims().items():
            if name in state_dict:
                state_dict[name] = self._gather_tp_tensor(state_dict[name], dim)

    def process_state_dict_for_loading(self, state_dict: dict[str, Any]) -> None:
        if self._tp_group is None:
            return
        for name, dim in self._tp_param_shard_dims().items():
            if name in state_dict and dim is not None:
                state_dict[name] = self._slice_tp_tensor(state_dict[name], dim)

    def process_named_optimizer_state_for_saving(self, optimizer_state: dict[str, dict[str, Any]]) -> None:
        if self._tp_group is None:
            return
        for name, dim in self._tp_param_shard_dims().items():
            st = optimizer_state.get(name)
            if st is None:
                continue
            for key, val in list(st.items()):
                if torch.is_tensor(val) and val.ndim > 0:
                    st[key] = self._gather_tp_tensor(val, dim)

    def process_named_optimizer_state_for_loading(self, optimizer_state: dict[str, dict[str, Any]]) -> None:
        if self._tp_group is None:
            return
        for name, dim in self._tp_param_shard_dims().items():
            st = optimizer_state.get(name)
            if st is None:
                continue
            for key, val in list(st.items()):
                if torch.is_tensor(val) and val.ndim > 0:
                    st[key] = self._slice_tp_tensor(val, dim)

    def sync_tensor_parallel_gradients(self) -> None:
        """Replicated params (b_dec) already hold identical full gradients on every rank
        (see `tp_copy`); the average keeps them bit-identical across ranks."""
        if self._tp_group is None:
            return
        _, size = self._tp_info()
        dims = self._tp_param_shard_dims()
        for name, p in self.named_parameters():
            if p.grad is None or dims.get(name) is not None:
                continue
            with nccl_nvtx_range("nccl:topk_tp_replicated_grad_all_reduce", self._tp_group):
                dist.all_reduce(p.grad, group=self._tp_group)
            p.grad /= size

    def clip_grad_norm_(self, max_norm: float, dp_group: dist.ProcessGroup | None = None) -> torch.Tensor:
        if self._tp_group is None and dp_group is None:
            return super().clip_grad_norm_(max_norm)
        rank, _ = self._tp_info()
        dims = self._tp_param_shard_dims()
        sq = torch.zeros((), device=self.W_dec.device, dtype=torch.float32)
        for name, p in self.named_parameters():
            if p.grad is None:
                continue
            g2 = p.grad.detach().float().pow(2).sum()
            if dims.get(name) is None:
                if rank == 0:
                    sq = sq + g2
            else:
                sq = sq + g2
        if self._tp_group is not None:
            with nccl_nvtx_range("nccl:topk_tp_grad_norm_all_reduce", self._tp_group):
                dist.all_reduce(sq, group=self._tp_group)
        if dp_group is not None:
            with nccl_nvtx_range("nccl:topk_dp_grad_norm_all_reduce", dp_group):
                dist.all_reduce(sq, group=dp_group)
        total = sq.sqrt()
        coef = (max_norm / (total + 1e-6)).clamp(max=1.0)
        for p in self.parameters():
            if p.grad is not None:
                p.grad.mul_(coef.to(device=p.grad.device, dtype=p.grad.dtype))
        return total

    def save_model(self, path: str | Path) -> tuple[Path, Path]:
        if self._tp_group is None:
            return super().save_model(path)
        return self._tp_save(path, inference=False)

    def save_inference_model(self, path: str | Path) -> tuple[Path, Path]:
        if self._tp_group is None:
            return super().save_inference_model(path)
        return self._tp_save(path, inference=True)

    def _tp_save(self, path: str | Path, inference: bool) -> tuple[Path, Path]:
        path = Path(path)
        path.mkdir(parents=True, exist_ok=True)
        sd = dict(self.state_dict())
        if inference:
            self.process_state_dict_for_saving_inference(sd)
            cfg_d = self.cfg.get_inference_sae_cfg_dict()
        else:
            self.process_state_dict_for_saving(sd)
            cfg_d = self.cfg.to_dict()
        wpath, cpath = path / SAE_WEIGHTS_FILENAME, path / SAE_CFG_FILENAME
        if dist.get_rank(self._tp_group) == 0:
            save_file({k: v.contiguous() for k, v in sd.items()}, wpath)
            with open(cpath, "w") as f:
                json.dump(cfg_d, f)
        with nccl_nvtx_range("nccl:topk_tp_save_barrier", self._tp_group):
            dist.barrier(group=self._tp_group)
        return wpath, cpath

    # ---------------------------------------------------------------- forward
    def encode_with_hidden_pre(self, x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        sae_in = tp_copy(self.process_sae_in(x), self._tp_group)
        pre_local = self.hook_sae_acts_pre(sae_in @ self.W_enc + self.b_enc)
        if self.cfg.rescale_acts_by_decoder_norm:
            pre_local = pre_local * self.W_dec.norm(dim=-1)
        pre = tp_allgather(pre_local, self._tp_group)
        return self.hook_sae_acts_post(self.activation_fn(pre)), pre

    def _local_slice(self, acts: torch.Tensor) -> torch.Tensor:
        rank, size = self._tp_info()
        n = acts.shape[-1] // size
        if acts.is_sparse:
            return acts.to_dense()[..., rank * n : (rank + 1) * n]
        return acts[..., rank * n : (rank + 1) * n]

    def decode(self, feature_acts: torch.Tensor) -> torch.Tensor:
        if self._tp_group is not None:
            local = self._local_slice(feature_acts)
            if self.cfg.rescale_acts_by_decoder_norm:
                local = local * (1 / self.W_dec.norm(dim=-1))
            out = tp_allreduce(local @ self.W_dec, self._tp_group) + self.b_dec
        else:
            out = act_times_W_dec(feature_acts, self.W_dec, self.cfg.rescale_acts_by_decoder_norm) + self.b_dec
        out = self.hook_sae_recons(out)
        out = self.run_time_activation_norm_fn_out(out)
        return self.reshape_fn_out(out, self.d_head)

    def calculate_aux_loss(self, step_input: TrainStepInput, feature_acts: torch.Tensor,
                           hidden_pre: torch.Tensor, sae_out: torch.Tensor) -> dict[str, torch.Tensor]:
        return {
            "auxiliary_reconstruction_loss": self.calculate_topk_aux_loss(
                sae_in=step_input.sae_in, sae_out=sae_out, hidden_pre=hidden_pre,
                dead_neuron_mask=step_input.dead_neuron_mask,
            )
        }

    def calculate_topk_aux_loss(self, sae_in: torch.Tensor, sae_out: torch.Tensor,
                                hidden_pre: torch.Tensor, dead_neuron_mask: torch.Tensor | None) -> torch.Tensor:
        if dead_neuron_mask is None or (num_dead := int(dead_neuron_mask.sum())) == 0:
            return sae_out.new_tensor(0.0)
        if self.cfg.normalize_activations in ("constant_norm_rescale", "layer_norm"):
            raise ValueError(
                "TopK auxiliary loss does not support activation normalization "
                f"(normalize_activations={self.cfg.normalize_activations!r})."
            )
        residual = (sae_in - sae_out).detach()
        k_aux = sae_in.shape[-1] // 2
        scale = min(num_dead / k_aux, 1.0)
        k_aux = min(k_aux, num_dead)
        aux_acts = calculate_topk_aux_acts(k_aux, hidden_pre, dead_neuron_mask)
        if self._tp_group is not None:
            local = self._local_slice(aux_acts)
            if self.cfg.rescale_acts_by_decoder_norm:
                local = local * (1 / self.W_dec.norm(dim=-1))
            recons = tp_allreduce(local @ self.W_dec, self._tp_group)
        else:
            recons = act_times_W_dec(aux_acts, self.W_dec, self.cfg.rescale_acts_by_decoder_norm)
        recons = self.reshape_fn_out(recons, self.d_head)
        loss = (recons - residual).pow(2).sum(dim=-1).mean()
        return self.cfg.aux_loss_coefficient * scale * loss

    @torch.no_grad()
    def fold_W_dec_norm(self) -> None:
        if not self.cfg.rescale_acts_by_decoder_norm:
            raise NotImplementedError(
                "Folding W_dec_norm is not safe for TopKSAEs when rescale_acts_by_decoder_norm is "
                "False, as this may change the topk activations"
            )
        _fold_norm_topk(self.W_enc, self.b_enc, self.W_dec)

    def process_state_dict_for_saving_inference(self, state_dict: dict[str, Any]) -> None:
        super().process_state_dict_for_saving_inference(state_dict)
        if self.cfg.rescale_acts_by_decoder_norm:
            W_enc = state_dict["W_enc"].clone()
            b_enc = state_dict["b_enc"].clone()
            W_dec = state_dict["W_dec"].clone()
            _fold_norm_topk(W_enc, b_enc, W_dec)
            state_dict["W_enc"], state_dict["b_enc"], state_dict["W_dec"] = W_enc, b_enc, W_dec
