"""Streaming mode of the LM training runner: producer GPUs run the LM and push activation chunks
into a ring, a disjoint consumer GPU set trains the SAE from it (behaviour of
sae_lens/llm_sae_training_runner.py:1112-1679 with sae_lens/distributed_streaming.py).

Two transports carry the chunks:

* "device" (default on CUDA with NCCL, SAE TP 1 and one hook): `DeviceActivationRing` in the
  consumer GPU's symmetric slab.  Producers claim slots over NVLink and store the rows with P2P
  stores, cast to bf16 in the same kernel; the consumer gathers batches on the device
  (`DeviceRingProvider`).  No host copy, no H2D.
* "host": the reference's design, a `/dev/shm` ring (`SharedActivationBuffer`) read by
  `StreamingActivationProvider` (pinned staging, async H2D, NCCL broadcast to SAE TP ranks).

Producers split the chunk quota statically (producer p writes sequence numbers p, p + P, ...),
watch the quiesce-request file between chunks (checkpoint their dataset position, then ack) and
signal "done" at the end.  The consumer trains through `SAETrainer` until the training tokens
are reached or every producer is done and the ring is empty.
"""

from __future__ import annotations

import math
import os
import time
from datetime import timedelta
from pathlib import Path
from typing import Any

import torch
import torch.distributed as dist

from saelens_b200.parallel import distributed_streaming as ds


def choose_transport(cfg: Any, sae_tp: int, n_hooks: int) -> str:
    want = getattr(cfg, "streaming_transport", "auto")
    if want != "auto":
        return want
    on_cuda = str(cfg.device).startswith("cuda") and torch.cuda.is_available()
    return "device" if (on_cuda and sae_tp == 1 and n_hooks == 1) else "host"


def streaming_init(runner: Any) -> None:
    """Process group, roles, and the ring (collective: every rank calls it)."""
    cfg = runner.cfg
    if not dist.is_initialized():
        backend = "nccl" if str(cfg.device).startswith("cuda") and torch.cuda.is_available() else "gloo"
        kw: dict[str, Any] = {}
        if backend == "nccl":
            local = int(os.environ.get("LOCAL_RANK", "0"))
            torch.cuda.set_device(local)
            kw["device_id"] = torch.device("cuda", local)
        # a short collective timeout: ranks left waiting on a rank that failed end with an error
        kw["timeout"] = timedelta(seconds=float(os.environ.get("SAELENS_B200_PG_TIMEOUT_S", "300")))
        dist.init_process_group(backend, **kw)
    vllm_tp, vllm_dp = max(runner.vllm_tp_size, 1), max(runner.vllm_dp_size, 1)
    sae_tp = max(runner.sae_tp_size, 1)
    ds.init_distributed_streaming(vllm_tp=vllm_tp, vllm_dp=vllm_dp, sae_tp=sae_tp, sae_dp=1)
    runner.role = "producer" if ds.is_producer() else "consumer"
    # the consumer ranks form one SAE tensor-parallel group: the runner shards the SAE over it
    runner.tp_group = ds.get_sae_tp_group() if sae_tp > 1 and not ds.is_producer() else None
    # producer tensor parallelism: every member runs the split LM, the group's first rank writes
    runner.producer_tp_group = ds.get_vllm_tp_group() if vllm_tp > 1 and ds.is_producer() else None
    runner.is_stream_writer = ds.is_producer() and ds.get_vllm_tp_rank() == 0
    n_hooks = len(getattr(cfg, "hook_names", None) or [cfg.hook_name])
    if n_hooks > 1 and cfg.streaming_chunk_size_tokens % cfg.train_batch_size_tokens:
        raise ValueError("multi-hook streaming needs streaming_chunk_size_tokens to be a multiple of "
                         "train_batch_size_tokens (chunks hold whole per-hook training batches)")
    runner.streaming_transport = choose_transport(cfg, sae_tp, n_hooks)
    runner.n_producers = vllm_dp
    runner.target_chunks = math.ceil(cfg.training_tokens / cfg.streaming_chunk_size_tokens)
    runner.ring = None
    runner.shm_buffer = None
    if runner.streaming_transport == "device":
        from saelens_b200.parallel.device_ring import DeviceActivationRing

        producers = [ds.get_producer_tp_root(p) for p in range(vllm_dp)]
        runner.ring = DeviceActivationRing(dist.group.WORLD, producers, ds.get_consumer_tp_root(0),
                                           n_slots=cfg.streaming_num_chunks,
                                           chunk_rows=cfg.streaming_chunk_size_tokens, d=cfg.sae.d_in)
    else:
        from saelens_b200.training.shared_activation_buffer import SharedActivationBuffer
        from saelens_b200.utils.misc import str_to_dtype

        name = cfg.streaming_buffer_name or f"saeb_{os.environ.get('MASTER_PORT', 'run')}_{os.getppid()}"
        kw = dict(name=name, num_chunks=cfg.streaming_num_chunks, chunk_size_tokens=cfg.streaming_chunk_size_tokens * n_hooks,
                  d_model=cfg.sae.d_in, num_producers=vllm_dp, target_chunks=runner.target_chunks,
                  base_dir=getattr(cfg, "streaming_buffer_dir", "/dev/shm"))
        exists = Path(kw["base_dir"], f"{name}.ctl").exists()
        if dist.get_rank() == 0 and not exists:  # fresh run; a restart attaches (READY chunks kept)
            dt = str_to_dtype(cfg.dtype)
            runner.shm_buffer = SharedActivationBuffer(
                create=True, dtype=dt if dt in (torch.bfloat16, torch.float32) else torch.bfloat16, **kw)
        dist.barrier()
        if runner.shm_buffer is None:
            runner.shm_buffer = SharedActivationBuffer(create=False, **kw)
        if str(cfg.device).startswith("cuda") and torch.cuda.is_available():
            # page-locked ring: producers copy device rows straight into their slot, the trainer
            # copies claimed slots straight to its GPU (no pageable host copy in between)
            runner.shm_buffer.register_for_device_copies()


def _quiesce_dir(runner: Any) -> Path | None:
    """Where quiesce requests and acks live: the supervisor's run directory when launched by it,
    else the checkpoint directory."""
    qdir = getattr(runner, "quiesce_dir", None)
    if qdir is None and runner.cfg.checkpoint_path is not None:
        qdir = runner.cfg.checkpoint_path
    return Path(qdir) if qdir is not None else None


def _quiesce_paths(runner: Any) -> tuple[Path | None, Path | None, Path | None]:
    qdir = _quiesce_dir(runner)
    if qdir is None:
        return None, None, None
    pidx = ds.get_producer_idx()
    return qdir / "quiesce_request", qdir / f"quiesce_ack_producer_{pidx}", qdir / f"producer_dataset_state_{pidx}"


def _hook_blocks(acts: torch.Tensor, n_hooks: int, batch: int) -> tuple[torch.Tensor, int]:
    """Multi-hook rows [n, H * d] (hooks side by side) as the ring's layout: per training step of
    `batch` tokens one block of `batch` rows per hook, [(n / batch) * H * batch, d]; a tail shorter
    than `batch` is dropped."""
    n = (acts.shape[0] // batch) * batch
    d = acts.shape[1] // n_hooks
    out = acts[:n].reshape(n // batch, batch, n_hooks, d).permute(0, 2, 1, 3).reshape(-1, d).contiguous()
    return out, int(out.shape[0])


def run_producer(runner: Any) -> int:
    """Write this producer's share of the chunk quota; returns the number of chunks written."""
    cfg, store = runner.cfg, runner.activations_store
    n_hooks = len(getattr(cfg, "hook_names", None) or [cfg.hook_name])
    pidx, P = ds.get_producer_idx(), runner.n_producers
    rows_per_chunk = cfg.streaming_chunk_size_tokens
    req, ack, state_dir = _quiesce_paths(runner)
    if runner.resume_from_checkpoint is not None and state_dir is not None and state_dir.exists():
        store.load_from_checkpoint(state_dir)  # continue this producer's dataset where it stopped
    def requested() -> bool:
        return req is not None and req.exists()

    def quiesce() -> None:
        if state_dir is not None:
            state_dir.mkdir(parents=True, exist_ok=True)
            store.save_to_checkpoint(state_dir)
        if ack is not None:
            ack.touch()

    writer = getattr(runner, "is_stream_writer", True)
    tp = getattr(runner, "producer_tp_group", None)
    written = 0
    seq = pidx
    if runner.ring is not None and runner.resume_from_checkpoint is not None:
        # the device ring starts empty after a restart: skip the chunks the consumer's checkpoint
        # already trained on (the /dev/shm ring keeps its own claim counter instead)
        from saelens_b200.constants import TRAINER_STATE_FILENAME

        st_path = Path(runner.resume_from_checkpoint) / TRAINER_STATE_FILENAME
        if st_path.exists():
            st = torch.load(st_path, map_location="cpu", weights_only=False)
            consumed = int(st.get("n_training_samples", 0)) // rows_per_chunk
            seq = pidx + ((max(consumed - pidx, 0) + P - 1) // P) * P
    stop = None  # None: go on; "quiesce": quiesce and stop; "end": the ring was closed
    while True:
        # the writer decides for its whole TP group (the members' LM forwards run in lockstep)
        go = seq < runner.target_chunks and stop is None and not (writer and requested())
        if tp is not None:
            flag = torch.tensor([1 if go else 0], dtype=torch.int32,
                                device="cuda" if dist.get_backend(tp) == "nccl" else "cpu")
            dist.broadcast(flag, src=dist.get_global_rank(tp, 0), group=tp)
            go = bool(flag.item())
        if not go:
            if writer and (stop == "quiesce" or (stop is None and seq < runner.target_chunks and requested())):
                quiesce()
            break
        rows = max(1, min(rows_per_chunk, cfg.training_tokens - seq * rows_per_chunk))
        acts, valid = store.get_streaming_activations(rows)
        if n_hooks > 1:
            acts, valid = _hook_blocks(acts, n_hooks, cfg.train_batch_size_tokens)
        if writer:
            # a full ring blocks the producer; the quiesce request must still reach it there
            if runner.ring is not None:
                if runner.ring.write(acts, stop_check=requested) is None:
                    stop = "quiesce"
                    continue
            else:
                buf = runner.shm_buffer
                got = buf.allocate_write_chunk(stop_check=requested)
                if got is None:
                    stop = "quiesce" if requested() else "end"
                    continue
                idx, _ = got
                buf.write_chunk(idx, acts.detach() if buf.registered else acts.detach().to("cpu"), valid,
                                producer_id=pidx)
                buf.mark_ready(idx)
            written += 1
        seq += P
    if writer:
        if runner.ring is not None:
            runner.ring.producer_done()
        else:
            runner.shm_buffer.signal_done()
    return written


class DeviceRingProvider:
    """Training batches from a `DeviceActivationRing` (consumer side).  Chunks are gathered on
    the device (rows permuted when `shuffle`), concatenated with the leftover of the previous
    chunk and cut into `train_batch_size_tokens` rows.  Stops when every producer is done and
    the ring holds no READY chunk."""

    def __init__(self, ring: Any, train_batch_size_tokens: int, shuffle: bool = True, seed: int = 0,
                 dtype: torch.dtype = torch.float32, timeout_s: float = 600.0):
        self.ring = ring
        self.batch = int(train_batch_size_tokens)
        self.shuffle = shuffle
        self.dtype = dtype
        self.timeout_s = timeout_s
        dev = ring.heap.device
        self._gen = torch.Generator(device=dev)
        self._gen.manual_seed(seed)
        self._pool: torch.Tensor | None = None
        self._consumed = 0

    def __iter__(self) -> DeviceRingProvider:
        return self

    @property
    def consumed_tokens(self) -> int:
        return self._consumed

    def _avail(self) -> int:
        return 0 if self._pool is None else self._pool.shape[0]

    def __next__(self) -> torch.Tensor:
        ring = self.ring
        while self._avail() < self.batch:
            t0 = time.monotonic()
            chunk = None
            while chunk is None:
                # done flags are set after a producer's last READY publish, so "done and nothing
                # READY" means the stream has ended
                if ring.producers_done() and ring.ready_chunks() == 0:
                    break
                try:
                    chunk, _ = ring.take(timeout_s=1.0, shuffle=self._gen if self.shuffle else None)
                except TimeoutError:
                    if time.monotonic() - t0 > self.timeout_s:
                        raise
            if chunk is None:
                break
            self._pool = chunk if self._pool is None else torch.cat([self._pool, chunk])
        if self._avail() == 0:
            raise StopIteration
        n = min(self.batch, self._avail())
        assert self._pool is not None
        b, self._pool = self._pool[:n], self._pool[n:]
        self._consumed += n
        return b.to(self.dtype)

    def consume_last_data_timing(self) -> dict[str, float]:
        return {"vllm_step_time_s": 0.0, "transfer_time_s": 0.0}


def run_consumer(runner: Any) -> Any:
    """Train the SAE from the ring; returns the trained SAE (on the consumer ranks)."""
    from saelens_b200.training.sae_trainer import SAETrainer
    from saelens_b200.training.streaming_activation_provider import StreamingActivationProvider
    from saelens_b200.utils.misc import str_to_dtype

    cfg = runner.cfg
    multi = bool(getattr(runner, "is_multi_sae", False))
    first = runner.base_sae_by_hook[runner.hook_names[0]] if multi else runner.sae
    dev = first.W_dec.device
    if runner.ring is not None:
        provider: Any = DeviceRingProvider(runner.ring, cfg.train_batch_size_tokens, shuffle=cfg.streaming_shuffle,
                                           seed=cfg.seed, dtype=str_to_dtype(cfg.dtype))
    else:
        tp = ds.get_sae_tp_group() if ds.get_sae_tp_size() > 1 else None
        provider = StreamingActivationProvider(
            runner.shm_buffer, cfg.train_batch_size_tokens, cfg.streaming_prefetch_chunks, dev, sae_tp_group=tp,
            sae_tp_rank=ds.get_sae_tp_rank(), sae_tp_root_global_rank=ds.get_consumer_tp_root(0),
            d_model=cfg.sae.d_in, dtype=str_to_dtype(cfg.dtype), shuffle=cfg.streaming_shuffle,
            random_chunks=cfg.streaming_random_chunks, hook_names=runner.hook_names if multi else None)
    qdir = _quiesce_dir(runner)
    if multi:
        return _run_multi_consumer(runner, provider, qdir)
    trainer = SAETrainer(cfg=cfg.to_sae_trainer_config(), sae=runner.sae, base_sae=runner.sae, data_provider=provider,
                         evaluator=None, save_checkpoint_fn=None,
                         append_logs=runner.resume_from_checkpoint is not None)
    runner.trainer = trainer
    if runner.resume_from_checkpoint is not None:
        ck = Path(runner.resume_from_checkpoint)
        runner.sae.load_weights_from_checkpoint(ck)
        if trainer.engine is not None:
            trainer.engine.refresh()
        trainer.load_trainer_state(ck)
    sae = trainer.fit(quiesce_request_path=qdir / "quiesce_request" if qdir is not None else None,
                      quiesce_ack_path=qdir / "quiesce_ack" if qdir is not None else None)
    if not getattr(trainer, "quiesced", False) and (runner.ring is None or ds.get_sae_tp_rank() == 0):
        runner.save_final_sae(sae, trainer)
    return sae


def _run_multi_consumer(runner: Any, provider: Any, qdir: Path | None) -> Any:
    """One SAE per hook from the ring's per-hook blocks (`MultiSAETrainer`); quiesce and resume as
    the single-hook consumer."""
    from saelens_b200.training.multi_sae_trainer import MultiSAETrainer

    cfg = runner.cfg
    trainer = MultiSAETrainer(
        hook_names=runner.hook_names, sae_by_hook=runner.sae_by_hook, base_sae_by_hook=runner.base_sae_by_hook,
        data_provider=provider, cfg=cfg.to_sae_trainer_config(), dp_group=None, sae_dp_mode=cfg.sae_dp_mode,
        backward_mode=cfg.multi_sae_backward_mode, seed_mode=cfg.multi_sae_seed_mode)
    runner.trainer = trainer
    if runner.resume_from_checkpoint is not None:
        trainer.load_trainer_state(runner.resume_from_checkpoint)
    result = trainer.fit(quiesce_request_path=qdir / "quiesce_request" if qdir is not None else None,
                         quiesce_ack_path=qdir / "quiesce_ack" if qdir is not None else None)
    if not trainer.quiesced and cfg.output_path is not None:
        trainer.save_final(cfg.output_path)  # every consumer rank (TP gathers), the first writes
    return result


def run_streaming(runner: Any) -> Any:
    """Entry point of `LanguageModelSAETrainingRunner.run()` in streaming mode."""
    result = None
    if runner.role == "producer":
        run_producer(runner)
    else:
        result = run_consumer(runner)
    dist.barrier()
    if runner.ring is not None:
        runner.ring.close()
    elif runner.shm_buffer is not None:
        runner.shm_buffer.close()
    return result


__all__ = ["DeviceRingProvider", "choose_transport", "run_consumer", "run_producer", "run_streaming",
           "streaming_init"]
