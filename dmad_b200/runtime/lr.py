"""Learning-rate schedules for the fused optimisers (which hold ``lr`` as an attribute).

Parity: diffusers ``get_scheduler`` names used by the H3 trainer (``constant``,
``constant_with_warmup``, ``linear``, ``cosine``; train/h3/lightx2v_train/trainers/base.py:74-80) and
the Wan stack's multi-cycle warm-up schedules (train/wan/rcm/utils/lr_scheduler.py:86-178):
``lambda_linear`` (its default: 100 warm-up steps from 1e-6 to 1, then constant 1,
configs/defaults/scheduler.py:22-28) and ``lambda_cosine``, with per-cycle ``warm_up_steps``,
``cycle_lengths``, ``f_start``, ``f_max`` and ``f_min``.
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


LAMBDA_LINEAR_DEFAULT = {"warm_up_steps": [100], "cycle_lengths": [10 ** 13], "f_start": [1.0e-6], "f_max": [1.0],
                         "f_min": [1.0]}


def lambda_factor(step: int, warm_up_steps, cycle_lengths, f_start, f_max, f_min, cosine: bool = False) -> float:
    """Multiplier of the multi-cycle schedules: the cycle is the first whose cumulative end is >= step;
    inside it, a linear warm-up from f_start to f_max, then linear (or cosine) decay to f_min at the
    cycle's end."""
    ends, acc = [], 0
    for c in cycle_lengths:
        acc += c
        ends.append(acc)
    cyc = next((i for i, e in enumerate(ends) if step <= e), len(ends) - 1)
    n = step - (ends[cyc - 1] if cyc > 0 else 0)
    W, L = warm_up_steps[cyc], cycle_lengths[cyc]
    if n < W:
        return (f_max[cyc] - f_start[cyc]) / W * n + f_start[cyc]
    if cosine:
        t = min((n - W) / (L - W), 1.0)
        return f_min[cyc] + 0.5 * (f_max[cyc] - f_min[cyc]) * (1 + math.cos(t * math.pi))
    return f_min[cyc] + (f_max[cyc] - f_min[cyc]) * (L - n) / (L - W)


class LRSchedule:
    def __init__(self, optimizer, name: str = "constant", warmup: int = 0, total: int = 1, f_min: float = 0.0,
                 cycles: dict | None = None):
        self.opt = optimizer
        self.name, self.warmup, self.total, self.f_min = name, int(warmup), int(total), float(f_min)
        self.cycles = dict(cycles or (LAMBDA_LINEAR_DEFAULT if name.startswith("lambda_") else {}))
        self.base_lr = float(optimizer.lr)
        self.step_num = 0
        self._apply()

    def factor(self, step: int) -> float:
        if self.name in ("lambda_linear", "lambda_cosine"):
            return lambda_factor(step, cosine=self.name == "lambda_cosine", **self.cycles)
        return lr_factor(self.name, step, self.warmup, self.total, f_min=self.f_min)

    def _apply(self):
        self.opt.lr = self.base_lr * self.factor(self.step_num)

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
