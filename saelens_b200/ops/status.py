"""Device status word shared by the native kernels.

Every bounded wait in the CUDA code writes a non-zero code here when it gives up (instead of
spinning forever); `check()` turns that into a Python exception.  Reading the word costs a
device sync, so hot loops check it only at coarse intervals.
"""

from __future__ import annotations

import torch

STATUS_MESSAGES = {
    0: "ok",
    1: "TMA producer timed out waiting for a free shared-memory stage",
    2: "MMA issuer timed out waiting for a loaded stage",
    3: "MMA issuer timed out waiting for a free TMEM accumulator",
    4: "epilogue timed out waiting for an accumulator",
    5: "timed out waiting for a peer flag",
    6: "top-k candidate buffer overflow",
}


class KernelTimeoutError(RuntimeError):
    pass


class StatusWord:
    def __init__(self, device: torch.device | str):
        self.tensor = torch.zeros(1, dtype=torch.int32, device=device)

    def code(self) -> int:
        return int(self.tensor.item())

    def check(self, where: str = "") -> None:
        c = self.code()
        if c != 0:
            self.tensor.zero_()
            raise KernelTimeoutError(
                f"{where}: native kernel reported status {c} ({STATUS_MESSAGES.get(c, 'unknown')})"
            )

    def reset(self) -> None:
        self.tensor.zero_()
