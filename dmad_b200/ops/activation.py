"""GELU (tanh approximation), as used by the Wan FFN and text embedding
(train/wan/rcm/networks/wan2pt1.py:386, 586)."""
from __future__ import annotations

import torch
import torch.nn.functional as F

from . import ext


class _Gelu(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x):
        y = torch.empty_like(x)
        ext().gelu_fwd(x, y)
        ctx.save_for_backward(x)
        return y

    @staticmethod
    def backward(ctx, g):
        (x,) = ctx.saved_tensors
        g = g.contiguous()
        dx = torch.empty_like(x)
        ext().gelu_bwd(g, x, dx)
        return dx


def gelu_tanh(x: torch.Tensor) -> torch.Tensor:
    if not x.is_cuda or x.dtype != torch.bfloat16 or x.numel() % 8:
        return F.gelu(x.float(), approximate="tanh").to(x.dtype)
    return _Gelu.apply(x.contiguous())
