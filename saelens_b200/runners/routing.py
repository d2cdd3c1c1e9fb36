"""Shard-routing mode of the LM training runner (`use_shard_routing=True`, the reference's v2
layout: sae_lens/distributed_v2.py:94-229 with sae_lens/training/activations_store.py:1351-1606).

P producers (each runs the LM on one GPU) and Q consumers (SAE replicas of `sae_tp` ranks) step in
lockstep.  Every step each producer makes `Q * train_batch / P` activation rows and the routing
table (`compute_routing_table`, interval overlap) splits them over the consumers; each consumer
trains on its assembled rows (earlier producers first).  A rank may be a producer, a consumer or
both.  With SAE TP every member of a consumer's TP group needs the same rows: the p2p transport
stores them into every member's landing buffer from the producer (no second hop), the collective
transport sends them to the consumer root, which broadcasts them to its TP group.

Several hooks (`hook_names`, one SAE per hook on every consumer): a producer's row carries the
hooks' activations side by side ([rows, n_hooks * d_in], every hook of the same width), so the
routing table, the router and the transports are the ones of a single hook with a wider row; the
consumer splits each received batch into one [rows, d_in] batch per hook for `MultiSAETrainer`.

Producer tensor parallelism (`vllm_tp_size` > 1): every member of a producer's TP group runs the
Megatron-split LM (`models/lm/tp.py`) on the same tokens in lockstep; the group's first rank holds
the full activations after the layer's all-reduces and is the one that sends.

Transports:

* "p2p" (CUDA + NCCL): `P2PRowRouter`, one kernel per producer step that stores every route's rows
  into the consumers' landing buffers over NVLink with the bf16 cast fused; the consumer reads its
  slot in place and releases it one step later (double buffering, producers throttled by the
  releases).  Long waits (an LM step, a consumer's first steps) happen on the host first, so the
  kernels' bounded waits find their data.
* "collective": `torch.distributed` point-to-point sends of the slices to the consumer roots
  (the reference's NCCL P2P exchange; also the CPU / gloo path).
"""

from __future__ import annotations

import math
import os
from pathlib import Path
from typing import Any

import torch
import torch.distributed as dist

from saelens_b200.parallel import distributed_v2 as v2

# host-side bound on one routed wait (an LM step, a slow consumer); SAELENS_B200_ROUTE_WAIT_S overrides
HOST_WAIT_S = float(os.environ.get("SAELENS_B200_ROUTE_WAIT_S", "600"))


def routing_init(runner: Any) -> None:
    """Process group, the v2 layout and roles, and the router (collective)."""
    cfg = runner.cfg
    if not dist.is_initialized():
        backend = "nccl" if str(cfg.device).startswith("cuda") and torch.cuda.is_available() else "gloo"
        if backend == "nccl":
            torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
        dist.init_process_group(backend)
    P, Q = max(runner.vllm_dp_size, 1), max(runner.sae_dp_size, 1)
    vtp, stp = max(runner.vllm_tp_size, 1), max(runner.sae_tp_size, 1)
    if (Q * cfg.train_batch_size_tokens) % P:
        raise ValueError("sae_dp_size * train_batch_size_tokens must be divisible by vllm_dp_size")
    runner.route_batch = Q * cfg.train_batch_size_tokens // P
    hook_names = getattr(cfg, "hook_names", None)
    runner.route_hooks = list(hook_names) if hook_names else [getattr(cfg, "hook_name", None)]
    runner.route_width = cfg.sae.d_in * len(runner.route_hooks)  # hooks side by side in one row
    world = dist.get_world_size()
    disjoint = world == P * vtp + Q * stp and world != max(P * vtp, Q * stp)
    v2.init_distributed_v2(P=P, Q=Q, vllm_tp_size=vtp, sae_tp_size=stp, batch_size=runner.route_batch,
                           disjoint=disjoint)
    # every member of a producer's TP group runs the (sharded) LM; its first rank sends the rows
    runner.is_route_producer = v2.is_producer()
    runner.is_route_sender = v2.is_producer() and v2.get_vllm_tp_rank() == 0
    runner.producer_tp_group = v2.get_vllm_tp_group() if vtp > 1 and v2.is_producer() else None
    runner.is_route_consumer = v2.is_consumer()
    runner.role = ("producer+consumer" if runner.is_route_producer and runner.is_route_consumer
                   else "producer" if runner.is_route_producer else "consumer" if runner.is_route_consumer else "idle")
    runner.tp_group = v2.get_sae_tp_group() if stp > 1 and runner.is_route_consumer else None
    runner.dp_group = v2.get_sae_dp_group() if Q > 1 and runner.is_route_consumer else None
    on_nccl = dist.get_backend() == "nccl"
    want = getattr(cfg, "routing_transport", "auto")
    runner.routing_transport = want if want != "auto" else ("p2p" if on_nccl else "collective")
    runner.router = None
    producers = [v2.get_producer_tp_root(p) for p in range(P)]
    consumers = [v2.get_consumer_tp_root(c) for c in range(Q)]
    runner.route_producers, runner.route_consumers = producers, consumers
    runner.route_to_members = False
    if runner.routing_transport == "p2p":
        from saelens_b200.parallel.row_router import P2PRowRouter

        members = None
        if stp > 1:
            layout = v2.get_layout()
            members = [list(layout.consumer_ranks[c]) for c in range(Q)]
            runner.route_to_members = True
        runner.router = P2PRowRouter(dist.group.WORLD, producers, consumers, runner.route_batch,
                                     runner.route_width, consumer_members=members)


class _RowSource:
    """`n` activation rows at a time from a store that yields fixed-size batches (a multi-hook
    store's {hook: rows} batches become rows with the hooks side by side, in `hooks` order)."""

    def __init__(self, store: Any, hooks: list[str] | None = None):
        self.store = store
        self.hooks = hooks
        self.rest: torch.Tensor | None = None

    def _next(self) -> torch.Tensor:
        b = next(self.store)
        if isinstance(b, dict):
            names = self.hooks or list(b)
            widths = {b[h].shape[-1] for h in names}
            if len(widths) != 1:
                raise ValueError(f"routed multi-hook runs need hooks of one width, got {sorted(widths)}")
            b = torch.cat([b[h] for h in names], dim=-1)
        return b

    def take(self, n: int) -> torch.Tensor:
        parts, have = [], 0
        if self.rest is not None and self.rest.shape[0]:
            parts.append(self.rest)
            have = self.rest.shape[0]
        while have < n:
            b = self._next()
            parts.append(b)
            have += b.shape[0]
        cat = torch.cat(parts) if len(parts) > 1 else parts[0]
        self.rest = cat[n:]
        return cat[:n]


class RoutedExchange:
    """One routed step on this rank: produce and send (producers), receive and assemble
    (consumers).  `step()` returns the consumer's batch (None on producer-only ranks)."""

    def __init__(self, runner: Any):
        from saelens_b200.utils.misc import str_to_dtype

        self.r = runner
        self.cfg = runner.cfg
        self.source = _RowSource(runner.activations_store, runner.route_hooks) if runner.is_route_producer else None
        self.width = runner.route_width
        self.routes = v2.get_routing_table()
        self.p_idx = v2.get_producer_idx() if runner.is_route_producer else -1
        self.c_idx = v2.get_consumer_idx() if runner.is_route_consumer else -1
        self.dtype = str_to_dtype(self.cfg.dtype)
        self.dev = torch.device(self.cfg.device if str(self.cfg.device) != "cuda" else f"cuda:{torch.cuda.current_device()}")
        self._pending_release = False
        self.rank = dist.get_rank()
        # producers save their dataset position where the consumers' trainer checkpoints: after
        # the same steps (same thresholds), into the same directory, so a resume restarts both
        self.done_steps = 0
        self.produced = 0
        self._thresholds: list[int] = []
        if self.source is not None and self.cfg.n_checkpoints > 0 and self.cfg.checkpoint_path is not None:
            total = self.cfg.total_training_tokens
            stride = math.ceil(total / (self.cfg.n_checkpoints + 1))
            self._thresholds = list(range(0, total, stride))[1:]

    def _after_produce(self) -> None:
        self.produced += 1
        n = (self.done_steps + self.produced) * self.cfg.train_batch_size_tokens
        while self._thresholds and n > self._thresholds[0]:
            d = Path(self.cfg.checkpoint_path) / str(n) / f"producer_dataset_state_{self.p_idx}"
            d.mkdir(parents=True, exist_ok=True)
            self.r.activations_store.save_to_checkpoint(d)
            self._thresholds.pop(0)

    def _produce(self) -> torch.Tensor | None:
        return self.source.take(self.r.route_batch) if self.source is not None else None

    def step(self) -> torch.Tensor | None:
        rows = self._produce()
        if rows is not None and not self.r.is_route_sender:
            rows = None  # a producer TP member: the group's first rank sends
        if rows is not None:
            self._after_produce()
        if self.r.router is not None:
            return self._step_p2p(rows)
        return self._step_collective(rows)

    def _step_p2p(self, rows: torch.Tensor | None) -> torch.Tensor | None:
        router = self.r.router
        if self._pending_release:  # the previous step's rows were consumed (stream order)
            router.release()
            self._pending_release = False
        if rows is not None:
            router.send(rows.to(self.dev), host_wait_s=HOST_WAIT_S)
        if self.r.route_to_members:  # every TP member receives the rows itself
            if self.c_idx < 0:
                return None
            got = router.recv(host_wait_s=HOST_WAIT_S)
            self._pending_release = True
            return got.to(self.dtype)
        if self.c_idx < 0 or self.rank != self.r.route_consumers[self.c_idx]:
            return self._bcast_tp(None)
        got = router.recv(host_wait_s=HOST_WAIT_S)
        self._pending_release = True
        return self._bcast_tp(got.to(self.dtype))

    def _step_collective(self, rows: torch.Tensor | None) -> torch.Tensor | None:
        ops: list[dist.P2POp] = []
        local: dict[int, torch.Tensor] = {}
        recv: dict[int, torch.Tensor] = {}
        is_root = self.c_idx >= 0 and self.rank == self.r.route_consumers[self.c_idx]
        d = self.width
        for rt in self.routes:
            src, dst = self.r.route_producers[rt.producer_idx], self.r.route_consumers[rt.consumer_idx]
            if rt.producer_idx == self.p_idx and rows is not None:
                piece = rows[rt.row_start : rt.row_end].to(self.dtype).contiguous()
                if dst == self.rank:
                    local[rt.producer_idx] = piece
                else:
                    ops.append(dist.P2POp(dist.isend, piece, dst))
            if is_root and rt.consumer_idx == self.c_idx and src != self.rank:
                buf = torch.empty(rt.row_end - rt.row_start, d, dtype=self.dtype, device=self.dev)
                recv[rt.producer_idx] = buf
                ops.append(dist.P2POp(dist.irecv, buf, src))
        if ops:
            for w in dist.batch_isend_irecv(ops):
                w.wait()
        if not is_root:
            return self._bcast_tp(None)
        parts = {**recv, **local}
        return self._bcast_tp(torch.cat([parts[p] for p in sorted(parts)]))

    def _bcast_tp(self, batch: torch.Tensor | None) -> torch.Tensor | None:
        """SAE TP: the consumer root's rows go to every TP member (replicated input)."""
        tp = self.r.tp_group
        if tp is None or self.c_idx < 0:
            return batch
        root = self.r.route_consumers[self.c_idx]
        if batch is None:
            batch = torch.empty(self.cfg.train_batch_size_tokens, self.width, dtype=self.dtype, device=self.dev)
        dist.broadcast(batch, src=root, group=tp)
        return batch

    def finish(self) -> None:
        if self.r.router is not None and self._pending_release:
            self.r.router.release()
            self._pending_release = False


class RoutedProvider:
    """DataProvider of a consumer rank: each `next()` is one routed step (with `hooks`, a
    {hook: [rows, d_in]} batch cut from the hooks-side-by-side rows)."""

    def __init__(self, exchange: RoutedExchange, n_steps: int, hooks: list[str] | None = None):
        self.ex = exchange
        self.left = n_steps
        self.hooks = hooks if hooks and len(hooks) > 1 else None

    def __iter__(self) -> RoutedProvider:
        return self

    def __next__(self) -> torch.Tensor:
        if self.left <= 0:
            raise StopIteration
        self.left -= 1
        batch = self.ex.step()
        assert batch is not None
        if self.hooks is None:
            return batch
        d = batch.shape[1] // len(self.hooks)
        return {h: batch[:, i * d:(i + 1) * d].contiguous() for i, h in enumerate(self.hooks)}


def resume_state(runner: Any, ex: RoutedExchange) -> int:
    """Steps already trained in the resume checkpoint (0 without one); the producer side reloads
    its dataset position from the checkpoint and skips the checkpoint thresholds already passed."""
    ck = runner.resume_from_checkpoint
    if ck is None:
        return 0
    from saelens_b200.constants import TRAINER_STATE_FILENAME

    st = torch.load(Path(ck) / TRAINER_STATE_FILENAME, map_location="cpu", weights_only=False)
    # samples, not the step counter: a checkpoint is written before its step is counted
    done = int(st.get("n_training_samples", 0)) // runner.cfg.train_batch_size_tokens
    ex.done_steps = done
    n_done = done * runner.cfg.train_batch_size_tokens
    ex._thresholds = [t for t in ex._thresholds if t >= n_done]
    if ex.source is not None:
        state = Path(ck) / f"producer_dataset_state_{ex.p_idx}"
        if state.exists():
            runner.activations_store.load_from_checkpoint(state)
    return done


def run_producer_only(runner: Any, n_steps: int) -> None:
    ex = RoutedExchange(runner)
    done = resume_state(runner, ex)
    for _ in range(n_steps - done):
        ex.step()
    ex.finish()


__all__ = ["RoutedExchange", "RoutedProvider", "resume_state", "routing_init", "run_producer_only"]
