"""Per-GPU memory model of a saelens_b200 training run (role of scripts/memory_model.py in the
reference, rebuilt for this framework's memory layout rather than fitted to measurements).

The native TopK engine keeps, per latent shard of N = d_sae / sae_tp latents and d = d_in:
  fp32 master W_dec, W_enc^T and their Adam moments      6 N d x 4 bytes
  bf16 compute copies of both                            2 N d x 2
  bf16 gradient rows of both                             2 N d x 2
  per-latent vectors (b_enc + moments, norms, bias, ...)  ~16 N x 4
and per step: the GEMM output buffer H (bf16, capped by `h_buffer_bytes`) with its 32- and
256-column maxima, top-k values/indices, decode outputs and the CSC pair lists.  Data parallelism
adds a second gradient buffer plus the all-reduce slab (landing area and result), tensor
parallelism the exchange slab (full input rows, candidate lists, fp32 partial rows, dL/dx_hat).
A producer LM adds its weights (split over producer TP ranks) and the activations of one forward.

Sharded data parallel (`fsdp=True`, the FSDP engine over `sae_dp` ranks) keeps masters, moments and
the reduced gradient rows for n = d_sae / sae_dp latents only, while the slab holds the full bf16
W_enc and W_dec (gathered inside the encoder GEMM) and S landing slots of n gradient rows per
matrix; H spans all d_sae latents.  The streaming ring (`ring_slots` x `ring_chunk_rows` bf16 rows)
and the row router's double-buffered landing slots (`route_rows` per step) are symmetric slabs,
allocated on every rank of their group.

CLI: `python -m saelens_b200.memory_model --d-in 4096 --d-sae 1048576 --k 128 --batch 16384 --sae-tp 8`.
"""

from __future__ import annotations

import argparse
import json
from dataclasses import asdict, dataclass

MB = 1 << 20


@dataclass
class MemoryEstimate:
    sae_state_mb: float
    step_buffers_mb: float
    parallel_slabs_mb: float
    producer_mb: float
    activation_buffer_mb: float
    runtime_mb: float

    @property
    def total_mb(self) -> float:
        return (self.sae_state_mb + self.step_buffers_mb + self.parallel_slabs_mb + self.producer_mb
                + self.activation_buffer_mb + self.runtime_mb)

    def to_dict(self) -> dict[str, float]:
        d = {k: round(v, 1) for k, v in asdict(self).items()}
        d["total_mb"] = round(self.total_mb, 1)
        return d


def estimate(*, d_in: int, d_sae: int, k: int, batch: int, sae_tp: int = 1, sae_dp: int = 1,
             h_buffer_bytes: int = 8 << 30, aux_k: int | None = None, producer_params: int = 0,
             producer_tp: int = 1, producer_dtype_bytes: int = 2, producer_tokens: int = 0,
             producer_d_model: int = 0, activation_buffer_rows: int = 0, fsdp: bool = False,
             ring_slots: int = 0, ring_chunk_rows: int = 0, route_rows: int = 0,
             runtime_mb: float = 600.0) -> MemoryEstimate:
    """Memory of one rank.  `batch` is the number of rows this rank's SAE group trains on per step
    (the tensor-parallel group shares it); `aux_k` > 0 includes the dead-latent aux buffers."""
    D = d_in
    if fsdp:
        if sae_tp != 1:
            raise ValueError("sharded data parallel does not combine with tensor parallelism")
        N = d_sae  # the step works on every latent; the state below is per shard
        n = d_sae // max(sae_dp, 1)
        state = 6 * n * D * 4 + 2 * n * D * 2 + 16 * n * 4 + 8 * D * 4 + 6 * N * 4
    else:
        N = d_sae // sae_tp
        state = 6 * N * D * 4 + 2 * N * D * 2 + 2 * N * D * 2 + 16 * N * 4 + 8 * D * 4
    rows_h = max(1, min(batch, (h_buffer_bytes // (2 * N)) // 128 * 128 or 128))
    h = rows_h * N * 2 * (1 + 1 / 16 + 1 / 128)
    kk = k
    topk = batch * kk * 8 * 2                      # values/indices (+ candidates scratch)
    decode = batch * D * (2 + 2 + 2) + batch * 4   # sae_out, dL/dx_hat, input copy, loss rows
    pairs = batch * kk * (8 + 12)                  # pair ids + (row, coef, dz)
    aux = 0
    if aux_k:
        aux = batch * aux_k * (8 + 8 + 20) + 2 * batch * D * 2
    step = h + topk + decode + pairs + aux
    slabs = 0.0
    if sae_tp > 1:
        S, Bo = sae_tp, batch // sae_tp
        slabs += batch * D * 2 + S * batch * kk * 8 + S * Bo * D * 4 + batch * D * 2 + batch * 16
        if aux_k:
            slabs += S * batch * aux_k * 8 + S * Bo * D * 4 + batch * D * 2
    if fsdp:
        slabs += 2 * N * D * 2 + 2 * N * D * 2 + 3 * N * 4 * 2  # full bf16 weights, landing slots, vectors
    elif sae_dp > 1:
        slabs += 2 * N * D * 2 * 3                  # local grads, landing area, averaged result
    slabs += ring_slots * ring_chunk_rows * D * 2
    slabs += 2 * route_rows * D * 2
    producer = 0.0
    if producer_params:
        producer += producer_params * producer_dtype_bytes / producer_tp
        producer += producer_tokens * producer_d_model * producer_dtype_bytes * 6  # live activations of a block
    act_buf = activation_buffer_rows * D * 2
    return MemoryEstimate(state / MB, step / MB, slabs / MB, producer / MB, act_buf / MB, runtime_mb)


def main() -> None:
    p = argparse.ArgumentParser(description="Per-GPU memory estimate of a saelens_b200 training run")
    p.add_argument("--d-in", type=int, default=4096)
    p.add_argument("--d-sae", type=int, default=1048576)
    p.add_argument("--k", type=int, default=128)
    p.add_argument("--batch", type=int, default=16384)
    p.add_argument("--sae-tp", type=int, default=1)
    p.add_argument("--sae-dp", type=int, default=1)
    p.add_argument("--aux-k", type=int, default=0)
    p.add_argument("--producer-params", type=int, default=0)
    p.add_argument("--producer-tp", type=int, default=1)
    p.add_argument("--producer-tokens", type=int, default=0)
    p.add_argument("--producer-d-model", type=int, default=0)
    p.add_argument("--activation-buffer-rows", type=int, default=0)
    p.add_argument("--fsdp", action="store_true", help="sharded data parallel over --sae-dp ranks")
    p.add_argument("--ring-slots", type=int, default=0)
    p.add_argument("--ring-chunk-rows", type=int, default=0)
    p.add_argument("--route-rows", type=int, default=0)
    a = p.parse_args()
    est = estimate(d_in=a.d_in, d_sae=a.d_sae, k=a.k, batch=a.batch, sae_tp=a.sae_tp, sae_dp=a.sae_dp,
                   aux_k=a.aux_k or None, producer_params=a.producer_params, producer_tp=a.producer_tp,
                   producer_tokens=a.producer_tokens, producer_d_model=a.producer_d_model,
                   activation_buffer_rows=a.activation_buffer_rows, fsdp=a.fsdp, ring_slots=a.ring_slots,
                   ring_chunk_rows=a.ring_chunk_rows, route_rows=a.route_rows)
    print(json.dumps(est.to_dict(), indent=2))


if __name__ == "__main__":
    main()
