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
    """GELU-tanh; the CPU path is the PyTorch restatement, the CUDA path is this package's kernel only
    (bf16, element count a multiple of 8: anything else on CUDA is an error, not a silent fallback)."""
    if not x.is_cuda:
        return F.gelu(x.float(), approximate="tanh").to(x.dtype)
    if x.dtype != torch.bfloat16 or x.numel() % 8:
        raise ValueError(f"gelu_tanh on CUDA takes bf16 tensors with numel % 8 == 0, got {x.dtype} "
                         f"with {x.numel()} elements")
    return _Gelu.apply(x.contiguous())
