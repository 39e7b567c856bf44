"""Learning-rate schedules (parity: astrai/trainer/schedule.py:47-235).

All three are ``torch.optim.lr_scheduler.LRScheduler`` subclasses whose extra
hyper-parameters round-trip through ``state_dict``:

* ``cosine``: linear warmup (floored at ``min_rate``) then cosine decay to
  ``min_rate`` over ``lr_decay_steps``;
* ``sgdr``: warmup then cosine restarts, cycle length multiplied by
  ``t_mult`` after each restart, rate in ``[min_rate, 1]``;
* ``wsd``: warmup, constant, then quadratic decay ``(1-min)(1-r)^2 + min``.
"""

from __future__ import annotations

import math
from abc import ABC, abstractmethod
from typing import Any, Dict, List

from torch.optim.lr_scheduler import LRScheduler

from astrai_b200.factory import Registry


class BaseScheduler(LRScheduler, ABC):
    _extra: tuple = ()

    @abstractmethod
    def get_lr(self) -> List[float]: ...

    def _factor(self) -> float:  # pragma: no cover - overridden
        return 1.0

    def state_dict(self) -> Dict[str, Any]:
        sd = super().state_dict()
        sd.update({k: getattr(self, k) for k in self._extra})
        return sd

    def load_state_dict(self, state_dict: Dict[str, Any]) -> None:
        sd = dict(state_dict)
        for k in self._extra:
            if k in sd:
                setattr(self, k, sd.pop(k))
        super().load_state_dict(sd)


class SchedulerFactory(Registry["BaseScheduler"]):
    pass


def _warmup(step: int, warmup: int, min_rate: float) -> float:
    return max(min_rate, step / max(warmup, 1))


@SchedulerFactory.register("cosine")
class CosineScheduler(BaseScheduler):
    _extra = ("warmup_steps", "lr_decay_steps", "min_rate", "total_steps")

    def __init__(self, optimizer, warmup_steps: int, lr_decay_steps: int, min_rate: float = 0.01, last_epoch: int = -1):
        self.warmup_steps, self.lr_decay_steps, self.min_rate = warmup_steps, lr_decay_steps, min_rate
        self.total_steps = warmup_steps + lr_decay_steps
        super().__init__(optimizer, last_epoch)

    def get_lr(self) -> List[float]:
        t = self.last_epoch
        if t < self.warmup_steps:
            f = _warmup(t, self.warmup_steps, self.min_rate)
        else:
            prog = min((t - self.warmup_steps) / max(self.lr_decay_steps, 1), 1.0)
            f = max(self.min_rate, 0.5 * (1.0 + math.cos(math.pi * prog)))
        return [b * f for b in self.base_lrs]


@SchedulerFactory.register("sgdr")
class SGDRScheduler(BaseScheduler):
    _extra = ("warmup_steps", "cycle_length", "min_rate", "t_mult")

    def __init__(self, optimizer, warmup_steps: int, cycle_length: int, min_rate: float = 0.01, t_mult: int = 2,
                 last_epoch: int = -1):
        self.warmup_steps, self.cycle_length, self.min_rate, self.t_mult = warmup_steps, cycle_length, min_rate, t_mult
        super().__init__(optimizer, last_epoch)

    def get_lr(self) -> List[float]:
        t = self.last_epoch
        if t < self.warmup_steps:
            return [b * _warmup(t, self.warmup_steps, self.min_rate) for b in self.base_lrs]
        since = t - self.warmup_steps
        length, done = self.cycle_length, 0
        while done + length <= since:
            done += length
            length *= self.t_mult
        cos = 0.5 * (1.0 + math.cos(math.pi * (since - done) / length))
        f = self.min_rate + (1.0 - self.min_rate) * cos
        return [b * f for b in self.base_lrs]


@SchedulerFactory.register("wsd")
class WSDScheduler(BaseScheduler):
    _extra = ("warmup_steps", "stable_steps", "decay_steps", "min_rate", "total_steps")

    def __init__(self, optimizer, warmup_steps: int, stable_steps: int, decay_steps: int, min_rate: float = 0.01,
                 last_epoch: int = -1):
        self.warmup_steps, self.stable_steps, self.decay_steps, self.min_rate = (warmup_steps, stable_steps,
                                                                                 decay_steps, min_rate)
        self.total_steps = warmup_steps + stable_steps + decay_steps
        super().__init__(optimizer, last_epoch)

    def get_lr(self) -> List[float]:
        t = self.last_epoch
        if t < self.warmup_steps:
            return [b * _warmup(t, self.warmup_steps, self.min_rate) for b in self.base_lrs]
        off = t - self.warmup_steps
        if off < self.stable_steps:
            return list(self.base_lrs)
        r = min((off - self.stable_steps) / max(self.decay_steps, 1), 1.0)
        f = (1.0 - self.min_rate) * (1.0 - r) ** 2 + self.min_rate
        return [b * f for b in self.base_lrs]
