"""Flash attention (forward + backward) on the sm_100a tcgen05 kernels.

Parity: ``attention(q, k, v)`` of the reference (train/wan/rcm/utils/attention.py:120-167),
layout ``[B, L, H, D]`` in and out, softmax scale ``1/sqrt(D)`` by default.
"""
from __future__ import annotations

import math
import os

import torch

from . import ext

# "split" (default): a dK/dV kernel and a dQ kernel, 7 GEMMs per tile pair, no atomics.
# "fused": one kernel for dK, dV and dQ (5 GEMMs; dQ through fp32 vector reductions into L2), used
# where the key tiles fill the GPU.  Measured on B200 at B=1, L=32760, H=12: split 21.3 ms, fused
# 26.2 ms -- the ~50 GB of dQ reductions per call cost more than the two GEMMs they save.
BWD_IMPL = os.environ.get("DMAD_FLASH_BWD", "split")
_FUSED_MIN_CTAS = 296  # two waves of the 148 SMs


def flash_bwd_into(q, k, v, o, do, lse, dq, dk, dv, dd, scale):
    """dq, dk, dv of softmax(q k^T scale) v given o, do and the forward's log2 LSE ([B, L, H, D] bf16 with
    D = 64 or 128, strided outputs allowed; ``dd`` an fp32 [B, H, Lpad] work buffer)."""
    e = ext()
    B, Lq, H, D = q.shape
    if BWD_IMPL == "fused" and D == 128 and -(-k.shape[1] // 128) * H * B >= _FUSED_MIN_CTAS:
        acc = torch.empty(B * H * lse.shape[-1] * 128, dtype=torch.float32, device=q.device)
        e.flash_bwd_fused(q, k, v, o, do, lse, dq, dk, dv, dd, acc, float(scale))
    else:
        e.flash_bwd(q, k, v, o, do, lse, dq, dk, dv, dd, float(scale))


def attention_reference(q, k, v, scale=None):
    """fp32 math of softmax(q k^T * scale) v on [B, L, H, D] tensors (oracle / CPU path)."""
    scale = scale if scale is not None else 1.0 / math.sqrt(q.shape[-1])
    qf, kf, vf = (t.float().transpose(1, 2) for t in (q, k, v))
    s = torch.matmul(qf, kf.transpose(-1, -2)) * scale
    p = torch.softmax(s, dim=-1)
    return torch.matmul(p, vf).transpose(1, 2).to(q.dtype)


def _lse_pad(L: int) -> int:
    return (L + 255) // 256 * 256


@torch.library.custom_op("dmad::flash_attn_fwd", mutates_args=(), device_types="cuda")
def flash_attn_fwd(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: float) -> tuple[torch.Tensor, torch.Tensor]:
    """(o [B, Lq, H, D] bf16, log2 LSE [B, H, round_up(Lq, 256)] fp32) of one tcgen05 forward.  A
    dispatcher op, so that selective activation checkpointing can keep its outputs."""
    B, Lq, H, D = q.shape
    o = torch.empty((B, Lq, H, D), dtype=q.dtype, device=q.device)
    lse = torch.empty((B, H, _lse_pad(Lq)), dtype=torch.float32, device=q.device)
    ext().flash_fwd(q, k, v, o, lse, float(scale))
    return o, lse


@flash_attn_fwd.register_fake
def _(q, k, v, scale):
    B, Lq, H, D = q.shape
    return q.new_empty((B, Lq, H, D)), q.new_empty((B, H, _lse_pad(Lq)), dtype=torch.float32)


class _FlashAttn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, scale):
        o, lse = flash_attn_fwd(q, k, v, float(scale))
        ctx.save_for_backward(q, k, v, o, lse)
        ctx.scale = scale
        return o

    @staticmethod
    def backward(ctx, do):
        q, k, v, o, lse = ctx.saved_tensors
        do = do.contiguous() if do.stride(-1) != 1 or do.stride(1) % 8 else do
        dq = torch.empty_like(q, memory_format=torch.contiguous_format)
        dk = torch.empty(k.shape, dtype=k.dtype, device=k.device)
        dv = torch.empty(v.shape, dtype=v.dtype, device=v.device)
        dd = torch.empty_like(lse)
        flash_bwd_into(q, k, v, o, do, lse, dq, dk, dv, dd, ctx.scale)
        return dq, dk, dv, None


def _supported(q, k, v, dims=(64, 128)) -> bool:
    return (q.is_cuda and q.shape[-1] in dims and q.dtype == torch.bfloat16 and k.dtype == q.dtype
            and v.dtype == q.dtype and k.shape[-1] == q.shape[-1] and v.shape[-1] == q.shape[-1])


def flash_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: float | None = None) -> torch.Tensor:
    """softmax(q k^T * scale) v for [B, L, H, D] bf16 tensors, D = 64 or 128 (strided views allowed).

    CUDA: sm_100a tcgen05 forward/backward kernels.  CPU: fp32 PyTorch math.
    """
    scale = float(scale) if scale is not None else 1.0 / math.sqrt(q.shape[-1])
    if not q.is_cuda:
        return attention_reference(q, k, v, scale)
    if not _supported(q, k, v):
        raise ValueError(f"flash_attention: need CUDA bf16 [B, L, H, 64 or 128], got {tuple(q.shape)} {q.dtype}")
    return _FlashAttn.apply(q, k, v, scale)


def _bhld_ok(t):
    return t.stride(-1) == 1 and all(s % 8 == 0 for s in t.stride()[:-1]) and t.data_ptr() % 16 == 0


class _FlashAttnJvp(torch.autograd.Function):
    """(O, tO) in one tcgen05 pass; the gradient flows through O only (tangents are detached), by
    the plain flash backward on the LSE the JVP kernel writes."""

    @staticmethod
    def forward(ctx, q, k, v, tq, tk, tv, scale):
        B, Lq, H, D = q.shape
        o = torch.empty((B, Lq, H, D), dtype=q.dtype, device=q.device)
        to = torch.empty_like(o)
        lse = torch.empty((B, H, _lse_pad(Lq)), dtype=torch.float32, device=q.device)
        fix = lambda t: t if t is None or _bhld_ok(t) else t.contiguous()  # noqa: E731
        tq, tk, tv = fix(tq.detach()), fix(tk.detach() if tk is not None else None), fix(
            tv.detach() if tv is not None else None)
        ext().flash_jvp_fwd(q, k, v, tq, tk, tv, o, to, lse, float(scale))
        ctx.save_for_backward(q, k, v, o, lse)
        ctx.scale = scale
        ctx.mark_non_differentiable(to)
        return o, to

    @staticmethod
    def backward(ctx, do, _dto):
        q, k, v, o, lse = ctx.saved_tensors
        do = do.contiguous() if do.stride(-1) != 1 or do.stride(1) % 8 else do
        dq = torch.empty_like(q, memory_format=torch.contiguous_format)
        dk = torch.empty(k.shape, dtype=k.dtype, device=k.device)
        dv = torch.empty(v.shape, dtype=v.dtype, device=v.device)
        dd = torch.empty_like(lse)
        flash_bwd_into(q, k, v, o, do, lse, dq, dk, dv, dd, ctx.scale)
        return dq, dk, dv, None, None, None, None


def attention_jvp_reference(q, k, v, tq, tk=None, tv=None, scale=None):
    """fp32 (O, tO) of softmax attention and its forward-mode tangent ([B, L, H, D]; oracle / CPU)."""
    scale = scale if scale is not None else 1.0 / math.sqrt(q.shape[-1])
    tr = lambda t: t.float().transpose(1, 2)  # noqa: E731
    qf, kf, vf, tqf = tr(q), tr(k), tr(v), tr(tq)
    s = qf @ kf.transpose(-1, -2) * scale
    ts = tqf @ kf.transpose(-1, -2)
    if tk is not None:
        ts = ts + qf @ tr(tk).transpose(-1, -2)
    ts = ts * scale
    p = torch.softmax(s, dim=-1)
    o = p @ vf
    pts = p * ts
    to = pts @ vf - pts.sum(-1, keepdim=True) * o
    if tv is not None:
        to = to + p @ tr(tv)
    return o.transpose(1, 2).to(q.dtype), to.transpose(1, 2).to(q.dtype)


def flash_attention_jvp(q, k, v, tq, tk=None, tv=None, scale: float | None = None):
    """(softmax(q k^T s) v, its tangent along (tq, tk, tv)) for [B, L, H, 128] bf16 tensors.

    CUDA: one sm_100a tcgen05 kernel (S, tS, O, A+B accumulators in TMEM); differentiable in O.
    CPU: fp32 PyTorch math.  ``tk`` / ``tv`` = None means a zero tangent (no GEMM is spent on it).
    """
    scale = float(scale) if scale is not None else 1.0 / math.sqrt(q.shape[-1])
    if not q.is_cuda:
        return attention_jvp_reference(q, k, v, tq, tk, tv, scale)
    if not _supported(q, k, v, dims=(128,)) or tq.dtype != q.dtype:
        raise ValueError(f"flash_attention_jvp: need CUDA bf16 [B, L, H, 128], got {tuple(q.shape)} {q.dtype}")
    return _FlashAttnJvp.apply(q, k, v, tq, tk, tv, scale)
