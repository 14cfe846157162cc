"""LoRA-fused linear on the persistent tcgen05 GEMM (csrc/gemm.cu).

    y = x W^T + bias + s (x A^T) (B o mask)^T

Forward = two launches of the same kernel: ``xa = s x A^T`` (N = r), then one GEMM over the
concatenated K panels ``[x | xa] [W | B o mask]^T`` with the bias in the epilogue.  Backward on the
same kernel, with operands read transposed in place (MN-major tiles) instead of materialised:
``g_s = s dY B`` (N = r), then ``dX = [dY | g_s] [W^T | A^T]^T`` as one GEMM over two K panels (the
forward's trick again), and the weight gradients ``dA = g_s^T x``, ``dB = dY^T xa`` (and ``dW = dY^T x``
when W trains) as split-K GEMMs over the token dimension (few output tiles, a long K: the K loop is
spread over the SMs and the fp32 partial sums are reduced in the epilogue).  Parity: PEFT's LoraLayer on
nn.Linear, as the reference's LoRA students use it (train/h3/lightx2v_train/model_zoo/base.py:16-114).
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
        g = _rows(gy).contiguous()
        e = ext()
        M, N = g.shape
        r, K = a.shape
        b = b.contiguous()
        gxa = torch.empty((M, r), dtype=g.dtype, device=g.device)   # s dY B
        e.gemm_bf16_ex(g, b, None, None, None, gxa, None, float(ctx.scale), 0, False, True, 1)
        dx = None
        if ctx.needs_input_grad[0]:
            dx = torch.empty((M, K), dtype=g.dtype, device=g.device)
            e.gemm_bf16_ex(g, w.contiguous(), gxa, a.contiguous(), None, dx, None, 1.0, 0, False, True, 1)
            dx = dx.view(ctx.xshape)
        da = _grad_gemm(gxa, x2) if ctx.needs_input_grad[3] else None    # [r, K] = g_s^T x
        db = _grad_gemm(g, xa) if ctx.needs_input_grad[4] else None      # [N, r] = dY^T xa
        dw = _grad_gemm(g, x2) if ctx.needs_input_grad[1] else None      # [N, K] = dY^T x
        dbias = g.float().sum(0).to(gy.dtype) if (ctx.has_bias and ctx.needs_input_grad[2]) else None
        return dx, dw, dbias, da, db, None


def _grad_gemm(p: torch.Tensor, q: torch.Tensor) -> torch.Tensor:
    """``p^T q`` for p [T, m], q [T, n] (T = tokens): both read MN-major; the T loop is split over enough
    CTAs to fill the GPU and the fp32 partial sums are reduced in the kernel's epilogue."""
    T, m = p.shape
    n = q.shape[1]
    tiles = -(-m // 128) * -(-n // 256)
    ksteps = -(-T // 64)
    sms = torch.cuda.get_device_properties(p.device).multi_processor_count
    split = max(1, min(ksteps // 4, -(-sms // tiles)))
    out = torch.zeros((m, n), dtype=torch.float32, device=p.device)
    ext().gemm_bf16_ex(p, q, None, None, None, None, out, 1.0, 0, True, True, split)
    return out.to(p.dtype)


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
