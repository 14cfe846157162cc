"""AdamW with fp32 master weights, driven by the multi-tensor sm_100a kernel.

Parity: the reference's ``FusedAdam(master_weights=True)`` / ``MasterWeightAdamW``
(train/wan/rcm/utils/fused_adam_dtensor.py:29-416): bf16 model weights, fp32 master
copies and fp32 moments, decoupled weight decay, bias correction.  One launch updates
a whole parameter group, writes the bf16 weights back, and (optionally) advances an
fp32 EMA copy of the weights in the same pass.
"""
from __future__ import annotations

import math
from typing import Iterable

import torch

from . import ext


class FusedAdamW:
    def __init__(self, params: Iterable[torch.nn.Parameter], lr=1e-4, betas=(0.9, 0.999), eps=1e-8,
                 weight_decay=0.0, ema: list[torch.Tensor] | None = None):
        self.params = [p for p in params]
        self.lr, self.betas, self.eps, self.weight_decay = lr, tuple(betas), eps, weight_decay
        self.step_count = 0
        self.master = [p.detach().float().clone() if p.dtype != torch.float32 else p.data for p in self.params]
        self.exp_avg = [torch.zeros_like(m) for m in self.master]
        self.exp_avg_sq = [torch.zeros_like(m) for m in self.master]
        self.ema = ema

    @property
    def param_groups(self):
        return [{"params": self.params, "lr": self.lr}]

    def zero_grad(self, set_to_none: bool = True):
        for p in self.params:
            if set_to_none:
                p.grad = None
            elif p.grad is not None:
                p.grad.zero_()

    def _lists(self, with_grad_only=True):
        idx = [i for i, p in enumerate(self.params) if p.grad is not None or not with_grad_only]
        return idx

    @torch.no_grad()
    def step(self, grad_scale: torch.Tensor | None = None, ema_beta: float | None = None,
             max_grad_norm: float | None = None):
        """One AdamW step.  ``grad_scale``: optional device scalar multiplied into the grads;
        ``max_grad_norm``: clip by the global gradient norm (computes ``grad_scale``).
        ``ema_beta``: when given (and an EMA list was attached), the EMA copies are advanced in
        the same kernel pass."""
        self.step_count += 1
        idx = self._lists()
        if not idx:
            return
        if grad_scale is None and max_grad_norm:
            grad_scale = clip_grad_scale([self.params[i] for i in idx], max_grad_norm)
        b1, b2 = self.betas
        on_cuda = self.params[idx[0]].is_cuda
        if not on_cuda:
            self._step_reference(idx, grad_scale, ema_beta)
            return
        # group by (grad dtype, has low-precision copy) so each launch is homogeneous
        groups: dict = {}
        for i in idx:
            p = self.params[i]
            key = (p.grad.dtype, p.dtype != torch.float32)
            groups.setdefault(key, []).append(i)
        for (gdt, has_lowp), ids in groups.items():
            grads = [self.params[i].grad.contiguous() for i in ids]
            master = [self.master[i] for i in ids]
            m = [self.exp_avg[i] for i in ids]
            v = [self.exp_avg_sq[i] for i in ids]
            lowp = [self.params[i].data for i in ids] if has_lowp else []
            ema = [self.ema[i] for i in ids] if (self.ema is not None and ema_beta is not None) else []
            ext().fused_adamw(master, grads, m, v, lowp, ema, float(self.lr), float(b1), float(b2), float(self.eps),
                              float(self.weight_decay), int(self.step_count), grad_scale,
                              float(ema_beta) if ema_beta is not None else 0.0)

    def _step_reference(self, idx, grad_scale, ema_beta):
        b1, b2 = self.betas
        bc1 = 1 - b1 ** self.step_count
        bc2 = 1 - b2 ** self.step_count
        gs = float(grad_scale) if grad_scale is not None else 1.0
        for i in idx:
            p = self.params[i]
            g = p.grad.float() * gs
            w = self.master[i]
            w.mul_(1 - self.lr * self.weight_decay)
            self.exp_avg[i].mul_(b1).add_(g, alpha=1 - b1)
            self.exp_avg_sq[i].mul_(b2).addcmul_(g, g, value=1 - b2)
            denom = (self.exp_avg_sq[i] / bc2).sqrt_().add_(self.eps)
            w.addcdiv_(self.exp_avg[i], denom, value=-self.lr / bc1)
            if p.dtype != torch.float32:
                p.data.copy_(w)
            if self.ema is not None and ema_beta is not None:
                self.ema[i].mul_(ema_beta).add_(w, alpha=1 - ema_beta)

    def state_dict(self):
        return {"step": self.step_count, "master": self.master, "exp_avg": self.exp_avg,
                "exp_avg_sq": self.exp_avg_sq, "lr": self.lr}

    def load_state_dict(self, sd):
        self.step_count = int(sd["step"])
        self.lr = sd.get("lr", self.lr)
        for dst, src in ((self.master, sd["master"]), (self.exp_avg, sd["exp_avg"]), (self.exp_avg_sq, sd["exp_avg_sq"])):
            for d, s in zip(dst, src):
                d.copy_(s)
        for p, m in zip(self.params, self.master):
            if p.dtype != torch.float32:
                p.data.copy_(m)


@torch.no_grad()
def clip_grad_scale(params, max_norm: float) -> torch.Tensor | None:
    """Device scalar min(1, max_norm / ||g||) (non-finite norm -> 0); None if clipping is off."""
    if max_norm is None or math.isinf(max_norm) or max_norm >= 1e11:
        return None
    grads = [p.grad.contiguous() for p in params if p.grad is not None]
    if not grads:
        return None
    dev = grads[0].device
    if not grads[0].is_cuda:
        n = torch.sqrt(sum((g.float() ** 2).sum() for g in grads))
        s = torch.clamp(max_norm / (n + 1e-6), max=1.0)
        return torch.where(torch.isfinite(n), s, torch.zeros_like(s))
    sumsq = torch.zeros(1, dtype=torch.float32, device=dev)
    by_dtype: dict = {}
    for g in grads:
        by_dtype.setdefault(g.dtype, []).append(g)
    for gl in by_dtype.values():
        ext().multi_sumsq(gl, sumsq)
    scale = torch.empty(1, dtype=torch.float32, device=dev)
    ext().clip_scale(sumsq, scale, float(max_norm))
    return scale
