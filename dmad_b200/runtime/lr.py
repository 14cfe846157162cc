"""Learning-rate schedules for the fused optimisers (which hold ``lr`` as an attribute).

Parity: diffusers ``get_scheduler`` names used by the H3 trainer (``constant``,
``constant_with_warmup``, ``linear``, ``cosine``; train/h3/lightx2v_train/trainers/base.py:74-80) and
the Wan ``LambdaLR`` warm-up / linear schedule (train/wan/rcm/utils/lr_scheduler.py:86-178).
"""
from __future__ import annotations

import math


def lr_factor(name: str, step: int, warmup: int, total: int, cycle_lengths=None, f_min: float = 0.0) -> float:
    if warmup > 0 and step < warmup:
        return (step + 1) / warmup if name != "constant" else 1.0
    if name in ("constant", "constant_with_warmup"):
        return 1.0
    progress = (step - warmup) / max(1, total - warmup)
    progress = min(max(progress, 0.0), 1.0)
    if name == "linear":
        return max(f_min, 1.0 - progress)
    if name == "cosine":
        return f_min + (1 - f_min) * 0.5 * (1.0 + math.cos(math.pi * progress))
    raise ValueError(f"unknown lr schedule {name!r}")


class LRSchedule:
    def __init__(self, optimizer, name: str = "constant", warmup: int = 0, total: int = 1, f_min: float = 0.0):
        self.opt = optimizer
        self.name, self.warmup, self.total, self.f_min = name, int(warmup), int(total), float(f_min)
        self.base_lr = float(optimizer.lr)
        self.step_num = 0
        self._apply()

    def _apply(self):
        self.opt.lr = self.base_lr * lr_factor(self.name, self.step_num, self.warmup, self.total, f_min=self.f_min)

    def step(self):
        self.step_num += 1
        self._apply()

    def get_last_lr(self):
        return [self.opt.lr]

    def state_dict(self):
        return {"step_num": self.step_num, "base_lr": self.base_lr, "name": self.name, "warmup": self.warmup,
                "total": self.total}

    def load_state_dict(self, sd):
        self.step_num = int(sd["step_num"])
        self.base_lr = float(sd["base_lr"])
        self._apply()
