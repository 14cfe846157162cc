"""LoRA-fused linear on the persistent tcgen05 GEMM (csrc/gemm.cu).

    y = x W^T + bias + s (x A^T) (B o mask)^T

Forward = two launches of the same kernel: ``xa = s x A^T`` (N = r), then one GEMM over the
concatenated K panels ``[x | xa] [W | B o mask]^T`` with the bias in the epilogue.  Backward uses
the library GEMMs (cuBLAS through torch): dX = dY W + (dY B) (s A), dA = s (dY B)^T x,
dB = dY^T xa, dW = dY^T x when W is trainable.  Parity: PEFT's LoraLayer on nn.Linear, as the
reference's LoRA students use it (train/h3/lightx2v_train/model_zoo/base.py:16-114).
"""
from __future__ import annotations

import torch

from . import ext


def _rows(t):
    return t.reshape(-1, t.shape[-1])


@torch.library.custom_op("dmad::lora_linear_fwd", mutates_args=(), device_types="cuda")
def lora_linear_fwd(x2: torch.Tensor, w: torch.Tensor, bias: torch.Tensor | None, a: torch.Tensor, b: torch.Tensor,
                    scale: float) -> tuple[torch.Tensor, torch.Tensor]:
    """(y, s x A^T) of the LoRA-fused linear on rows ``x2``.  A dispatcher op, so that selective
    activation checkpointing can keep its outputs."""
    M, N, r = x2.shape[0], w.shape[0], a.shape[0]
    e = ext()
    xa = torch.empty((M, r), dtype=x2.dtype, device=x2.device)
    e.gemm_bf16(x2, a.contiguous(), None, None, None, xa, float(scale), 0)
    y = torch.empty((M, N), dtype=x2.dtype, device=x2.device)
    e.gemm_bf16(x2, w.contiguous(), xa, b.contiguous(), bias.float().contiguous() if bias is not None else None,
                y, 1.0, 0)
    return y, xa


@lora_linear_fwd.register_fake
def _(x2, w, bias, a, b, scale):
    return x2.new_empty((x2.shape[0], w.shape[0])), x2.new_empty((x2.shape[0], a.shape[0]))


class _LoraLinear(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, bias, a, b, scale):
        x2 = _rows(x)
        x2 = x2 if (x2.stride(-1) == 1 and x2.stride(0) % 8 == 0) else x2.contiguous()
        N = w.shape[0]
        y, xa = lora_linear_fwd(x2, w, bias, a, b, float(scale))
        ctx.save_for_backward(x2, w, a, b, xa)
        ctx.scale = scale
        ctx.has_bias = bias is not None
        ctx.xshape = x.shape
        return y.view(*x.shape[:-1], N)

    @staticmethod
    def backward(ctx, gy):
        x2, w, a, b, xa = ctx.saved_tensors
        g = _rows(gy)
        gxa = g @ b                                   # [M, r]
        dx = g @ w + (gxa * ctx.scale) @ a
        da = (gxa.t() @ x2) * ctx.scale if ctx.needs_input_grad[3] else None
        db = g.t() @ xa if ctx.needs_input_grad[4] else None
        dw = g.t() @ x2 if ctx.needs_input_grad[1] else None
        dbias = g.float().sum(0).to(gy.dtype) if (ctx.has_bias and ctx.needs_input_grad[2]) else None
        return dx.view(ctx.xshape), dw, dbias, da, db, None


def lora_linear(x, w, bias, a, b, scale: float):
    """``x W^T + bias + scale (x A^T) B^T`` (B already masked for fused segments)."""
    if not x.is_cuda:
        y = torch.nn.functional.linear(x, w, bias)
        return y + scale * torch.nn.functional.linear(torch.nn.functional.linear(x, a), b)
    return _LoraLinear.apply(x, w, bias, a, b, float(scale))


def gemm(x, w, bias=None, act: str | None = None, alpha: float = 1.0):
    """``act(alpha * x W^T + bias)`` on the tcgen05 GEMM (forward only; for inference paths)."""
    x2 = _rows(x)
    y = torch.empty((x2.shape[0], w.shape[0]), dtype=x.dtype, device=x.device)
    ext().gemm_bf16(x2.contiguous(), w.contiguous(), None, None, bias.float().contiguous() if bias is not None
                    else None, y, float(alpha), {None: 0, "gelu_tanh": 1}[act])
    return y.view(*x.shape[:-1], w.shape[0])
