"""Legacy m:1 / mn:m fan-in data path of the LM training runner (`vllm_dp_size` = n * `sae_dp_size`
without shard routing; sae_lens/distributed.py:150-207 with
sae_lens/training/activations_store.py:1092-1279).

Each cluster of n ranks has one SAE root (cluster rank 0, also a producer) and n - 1 helper
producers.  After each of its own LM batches the root asks every helper for one batch over the
CPU (Gloo) group: a control word (1 = send a batch, 0 = stop), then the batch shape and rows.  The
root's mixing buffer receives its own and the helpers' batches in that order; at the end the
root sends 0 to every helper.  The exchange is a request / response, so a helper never sends
unasked and nothing waits on a message that is not coming.
"""

from __future__ import annotations

from typing import Any

import torch
import torch.distributed as dist


class FanInRoot:
    """Splices the helpers' batches into the root store's stream of LM batches."""

    def __init__(self, store: Any, helpers: list[int], group: dist.ProcessGroup):
        self.store, self.helpers, self.group = store, list(helpers), group
        self.received = 0
        own = store._llm_batches

        def batches() -> Any:
            for b in own():
                yield b
                for h in self.helpers:
                    yield self._fetch(h)

        store._llm_batches = batches

    def _fetch(self, helper: int) -> torch.Tensor:
        dist.send(torch.ones(1, dtype=torch.int64), helper, group=self.group)
        shape = torch.empty(2, dtype=torch.int64)
        dist.recv(shape, helper, group=self.group)
        buf = torch.empty(int(shape[0]), int(shape[1]), dtype=torch.float32)
        dist.recv(buf, helper, group=self.group)
        self.received += 1
        return buf.to(device=self.store.device, dtype=self.store.dtype)

    def close(self) -> None:
        for h in self.helpers:
            dist.send(torch.zeros(1, dtype=torch.int64), h, group=self.group)


def run_helper(store: Any, root: int, group: dist.ProcessGroup) -> int:
    """Serve the root's requests until it says stop; returns the number of batches sent."""
    sent = 0
    ctrl = torch.empty(1, dtype=torch.int64)
    while True:
        dist.recv(ctrl, root, group=group)
        if int(ctrl.item()) == 0:
            return sent
        b = store.get_filtered_llm_batch()
        if isinstance(b, dict):
            raise ValueError("the fan-in data path carries single-hook batches")
        b = b.detach().to("cpu", torch.float32).contiguous()
        dist.send(torch.tensor(list(b.shape), dtype=torch.int64), root, group=group)
        dist.send(b, root, group=group)
        sent += 1


__all__ = ["FanInRoot", "run_helper"]
