"""Learning-rate and loss-coefficient schedules (behaviour of sae_lens/training/optim.py).

`get_lr_scheduler` chains an optional linear warm-up, the main schedule (constant, cosine
annealing, cosine annealing with warm restarts) and an optional linear decay to zero.
`LRSchedule` evaluates the same curve as a pure function of the step, which the fused native
optimizer needs because it holds no torch optimizer.
"""

from __future__ import annotations

import math
from typing import Any

import torch.optim as optim
import torch.optim.lr_scheduler as lr_scheduler


def _main_scheduler(name: str, opt: optim.Optimizer, steps: int, lr_end: float, num_cycles: int):
    if name == "constant":
        return lr_scheduler.LambdaLR(opt, lr_lambda=lambda _s: 1.0)
    if name == "cosineannealing":
        return lr_scheduler.CosineAnnealingLR(opt, T_max=steps, eta_min=lr_end)
    if name == "cosineannealingwarmrestarts":
        return lr_scheduler.CosineAnnealingWarmRestarts(opt, T_0=steps // num_cycles, eta_min=lr_end)
    raise ValueError(f"Unsupported scheduler: {name}")


def get_lr_scheduler(scheduler_name: str, optimizer: optim.Optimizer, training_steps: int, lr: float,
                     warm_up_steps: int, decay_steps: int, lr_end: float, num_cycles: int) -> lr_scheduler.LRScheduler:
    name = scheduler_name.lower()
    main = _main_scheduler(name, optimizer, training_steps - warm_up_steps - decay_steps, lr_end, num_cycles)
    if name == "constant":
        lr_end = lr
    scheds: list[lr_scheduler.LRScheduler] = []
    milestones: list[int] = []
    if warm_up_steps > 0:
        scheds.append(lr_scheduler.LinearLR(optimizer, start_factor=1 / warm_up_steps, end_factor=1.0,
                                            total_iters=warm_up_steps - 1))
        milestones.append(warm_up_steps)
    scheds.append(main)
    if decay_steps > 0:
        if lr_end == 0.0:
            raise ValueError("Cannot have decay_steps with lr_end=0.0, this would decay from 0 to 0 and be a waste.")
        scheds.append(lr_scheduler.LinearLR(optimizer, start_factor=lr_end / lr, end_factor=0.0,
                                            total_iters=decay_steps))
        milestones.append(training_steps - decay_steps)
    return lr_scheduler.SequentialLR(optimizer, schedulers=scheds, milestones=milestones)


class LRSchedule:
    """The `get_lr_scheduler` curve without an optimizer: `lr_at(step)` for step 0, 1, ...

    It is validated against the torch scheduler chain in the tests; `state_dict` holds the step.
    """

    def __init__(self, scheduler_name: str, training_steps: int, lr: float, warm_up_steps: int,
                 decay_steps: int, lr_end: float, num_cycles: int):
        self.name = scheduler_name.lower()
        if self.name not in ("constant", "cosineannealing", "cosineannealingwarmrestarts"):
            raise ValueError(f"Unsupported scheduler: {scheduler_name}")
        self.training_steps = training_steps
        self.lr = lr
        self.warm = warm_up_steps
        self.decay = decay_steps
        self.lr_end = lr if self.name == "constant" else lr_end
        self.cosine_end = lr_end
        self.cycles = num_cycles
        if decay_steps > 0 and self.lr_end == 0.0:
            raise ValueError("Cannot have decay_steps with lr_end=0.0, this would decay from 0 to 0 and be a waste.")
        self.step_count = 0

    def _main(self, t: int) -> float:
        steps = self.training_steps - self.warm - self.decay
        if self.name == "constant":
            return self.lr
        if self.name == "cosineannealing":
            T = max(steps, 1)
            return self.cosine_end + (self.lr - self.cosine_end) * (1 + math.cos(math.pi * t / T)) / 2
        T0 = max(steps // self.cycles, 1)
        tc = t % T0
        return self.cosine_end + (self.lr - self.cosine_end) * (1 + math.cos(math.pi * tc / T0)) / 2

    def lr_at(self, step: int) -> float:
        if self.warm > 0 and step < self.warm:
            total = max(self.warm - 1, 1)
            frac = min(step, total) / total if self.warm > 1 else 1.0
            return self.lr * (1 / self.warm + (1 - 1 / self.warm) * frac)
        decay_start = self.training_steps - self.decay
        if self.decay > 0 and step >= decay_start:
            t = min(step - decay_start, self.decay)
            start = self.lr_end / self.lr
            return self.lr * (start + (0.0 - start) * t / self.decay)
        return self._main(step - self.warm)

    def get_last_lr(self) -> list[float]:
        return [self.lr_at(self.step_count)]

    def step(self) -> None:
        self.step_count += 1

    def state_dict(self) -> dict[str, Any]:
        return {"step_count": self.step_count}

    def load_state_dict(self, sd: dict[str, Any]) -> None:
        self.step_count = int(sd.get("step_count", sd.get("last_epoch", 0)))


class CoefficientScheduler:
    """Linear warm-up of a loss coefficient from 0 to `final_value`."""

    def __init__(self, warm_up_steps: float, final_value: float):
        self.warm_up_steps = warm_up_steps
        self.final_value = final_value
        self.current_step = 0
        if not isinstance(final_value, (float, int)):
            raise TypeError(f"final_value must be float or int, got {type(final_value)}.")
        self.current_value = 0.0 if warm_up_steps > 0 else final_value

    def __repr__(self) -> str:
        return f"{self.__class__.__name__}(final_value={self.final_value}, warm_up_steps={self.warm_up_steps})"

    def step(self) -> float:
        if self.current_step < self.warm_up_steps:
            self.current_value = self.final_value * ((self.current_step + 1) / self.warm_up_steps)
        else:
            self.current_value = self.final_value
        self.current_step += 1
        return self.current_value

    @property
    def value(self) -> float:
        return self.current_value

    def state_dict(self) -> dict[str, Any]:
        return {"current_step": self.current_step}

    def load_state_dict(self, sd: dict[str, Any]) -> None:
        for k, v in sd.items():
            setattr(self, k, v)
