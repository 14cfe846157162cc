"""Exponential moving averages of the generator.

* Power EMA (Karras et al., "Analyzing and improving the training dynamics of diffusion models"):
  beta_t = (1 - 1/t)^(gamma + 1).  The H3 trainer keeps two banks with gamma 6.94 and 16.97
  (train/h3/lightx2v_train/trainers/dmd/minimax_h3_dmad_trainer.py:458-480); the Wan model derives
  gamma from the relative width sigma_rel by the largest real root of t^3 + 7t^2 + (16 - s^-2)t + 12 - s^-2
  (train/wan/rcm/models/t2v_model_distill_rcm.py:270-277, 1149-1163).
* kimg half-life EMA with ramp-up for the EDM image trainer (train/image/main/edm/train_edm.py:176-184).
"""
from __future__ import annotations

import numpy as np
import torch


def ema_exp_coefficient(sigma_rel: float) -> float:
    s = sigma_rel
    return float(np.roots([1, 7, 16 - s ** -2, 12 - s ** -2]).real.max())


def power_ema_beta(t: int, gamma: float) -> float:
    """beta for the t-th update (t >= 1); t < 1 returns 0 (copy)."""
    if t < 1:
        return 0.0
    return (1.0 - 1.0 / t) ** (gamma + 1.0)


def kimg_halflife_beta(batch_size: int, cur_nimg: int, ema_halflife_kimg: float, ema_rampup_ratio: float | None):
    halflife = ema_halflife_kimg * 1000
    if ema_rampup_ratio is not None:
        halflife = min(halflife, cur_nimg * ema_rampup_ratio)
    return 0.5 ** (batch_size / max(halflife, 1e-8))


class PowerEMA:
    """fp32 shadow copies of a parameter list, updated with the power-EMA schedule."""

    def __init__(self, params, gamma: float):
        self.params = list(params)
        self.gamma = gamma
        self.shadow = [p.detach().float().clone() for p in self.params]
        self.t = 0

    @torch.no_grad()
    def update(self):
        self.t += 1
        beta = power_ema_beta(self.t, self.gamma)
        if self.shadow and self.shadow[0].is_cuda:
            torch._foreach_mul_(self.shadow, beta)
            torch._foreach_add_(self.shadow, [p.detach().float() for p in self.params], alpha=1.0 - beta)
        else:
            for s, p in zip(self.shadow, self.params):
                s.mul_(beta).add_(p.detach().float(), alpha=1.0 - beta)
        return beta

    def state_dict(self):
        return {"t": self.t, "gamma": self.gamma, "shadow": [s.cpu() for s in self.shadow]}

    def load_state_dict(self, sd):
        self.t = sd["t"]
        self.gamma = sd["gamma"]
        for s, v in zip(self.shadow, sd["shadow"]):
            s.copy_(v)
