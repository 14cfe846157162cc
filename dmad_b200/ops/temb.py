"""Timestep embedding: fp64 sinusoid and the small-M linear layers of the
modulation MLP (train/wan/rcm/networks/wan2pt1.py:181-190, 590-591, 772-784).

The forward runs the weight-streaming kernels of csrc/temb.cu; the backward of
these tiny-M layers is a pair of matmuls in PyTorch.
"""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F

from . import ext


def sinusoidal_embedding(t: torch.Tensor, dim: int, max_period: float = 10000.0) -> torch.Tensor:
    """[M] timesteps -> [M, dim] fp32 = cat(cos(t f), sin(t f)), f_j = max_period^(-j/(dim/2)), fp64 phases."""
    t = t.reshape(-1)
    if not t.is_cuda:
        half = dim // 2
        pos = t.double()
        freqs = torch.pow(torch.tensor(max_period, dtype=torch.float64), -torch.arange(half, dtype=torch.float64) / half)
        ph = torch.outer(pos, freqs.to(pos.device))
        return torch.cat([torch.cos(ph), torch.sin(ph)], dim=1).float()
    out = torch.empty((t.numel(), dim), dtype=torch.float32, device=t.device)
    ext().sinusoid_embed(t.float().contiguous(), out, int(dim), float(max_period))
    return out


class _SmallLinear(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, b, act_in):
        M = x.shape[0]
        y = torch.empty((M, w.shape[0]), dtype=torch.float32, device=x.device)
        ext().small_linear(x, w, b, y, int(act_in))
        ctx.save_for_backward(x, w)
        ctx.act_in = act_in
        ctx.has_b = b is not None
        return y

    @staticmethod
    def backward(ctx, gy):
        x, w = ctx.saved_tensors
        xa = F.silu(x) if ctx.act_in == 1 else x
        gx = gy @ w.float()
        if ctx.act_in == 1:
            s = torch.sigmoid(x)
            gx = gx * (s * (1 + x * (1 - s)))
        gw = (gy.t() @ xa).to(w.dtype) if ctx.needs_input_grad[1] else None
        gb = gy.sum(0) if ctx.has_b and ctx.needs_input_grad[2] else None
        return gx, gw, gb, None


def small_linear(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None, act_in: str | None = None):
    """fp32 y = act_in(x) @ weight^T + bias for a handful of rows (M <= 16)."""
    a = 1 if act_in == "silu" else 0
    if not x.is_cuda or x.shape[0] > 16 or weight.dtype != torch.bfloat16 or weight.shape[1] % 8:
        xa = F.silu(x.float()) if a == 1 else x.float()
        return F.linear(xa, weight.float(), bias.float() if bias is not None else None)
    return _SmallLinear.apply(x.float().contiguous(), weight.contiguous(), bias.float() if bias is not None else None, a)
