"""Normalisation, modulation, gated residual and RoPE ops.

Row tensors are 2-D ``[R, D]`` (rows contiguous, any row stride).  Per-row
modulation tensors are ``[G, D]`` fp32 and a row ``r`` uses group
``r // rows_per_group`` (or ``gidx[r]`` when an explicit int32 index is given,
as in the packed H3 layout, dmad_h3/lowmem.py:436-438).

Parity:
* ``ln_mod``: ``WanLayerNorm(x) * (1 + scale) + shift`` (train/wan/rcm/networks/wan2pt1.py:214-224, 419-436),
  affine ``nn.LayerNorm`` (cross-attention norm3) and ``WanRMSNorm`` (wan2pt1.py:193-211).
* ``gate_residual``: ``x + y * gate`` (wan2pt1.py:426-436).
* ``qk_norm_rope``: RMSNorm of q and k over the hidden size, then interleaved RoPE
  (rcm/utils/rope.py:36-70 with the frequency layout of wan2pt1.py:62-179).
"""
from __future__ import annotations

import torch

from . import ext

# ----------------------------------------------------------------------------- reference math


def _groups(R: int, rows_per_group: int, gidx):
    if gidx is not None:
        return gidx.long()
    return torch.arange(R, device=gidx.device if gidx is not None else None) // max(1, rows_per_group)


def ln_mod_reference(x, a=None, c=None, a_add=1.0, rows_per_group=None, gidx=None, eps=1e-6, rms=False):
    xf = x.float()
    if rms:
        n = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    else:
        mu = xf.mean(-1, keepdim=True)
        n = (xf - mu) * torch.rsqrt((xf - mu).pow(2).mean(-1, keepdim=True) + eps)
    R = x.shape[0]
    rpg = rows_per_group if rows_per_group is not None else R
    g = gidx.long().to(x.device) if gidx is not None else torch.arange(R, device=x.device) // max(1, rpg)
    A = a_add + (a.float()[g] if a is not None else 0.0)
    C = c.float()[g] if c is not None else 0.0
    return (n * A + C).to(x.dtype)


# ----------------------------------------------------------------------------- ln_mod


def _opt(t):
    return t if t is not None else None


class _LnMod(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, a, c, a_add, rows_per_group, gidx, eps, rms):
        R, D = x.shape
        y = torch.empty((R, D), dtype=x.dtype, device=x.device)
        rstd = torch.empty(R, dtype=torch.float32, device=x.device)
        mean = None if rms else torch.empty(R, dtype=torch.float32, device=x.device)
        ext().ln_mod_fwd(x, y, mean, rstd, a, c, float(a_add), int(rows_per_group), gidx, float(eps), bool(rms))
        ctx.save_for_backward(x, mean, rstd, a, gidx)
        ctx.cfg = (float(a_add), int(rows_per_group), bool(rms), c is not None, a is not None and a.requires_grad,
                   a.shape if a is not None else None, c.shape if c is not None else None)
        return y

    @staticmethod
    def backward(ctx, dy):
        x, mean, rstd, a, gidx = ctx.saved_tensors
        a_add, rpg, rms, has_c, _, a_shape, c_shape = ctx.cfg
        if dy.stride(-1) != 1 or dy.stride(0) % 8:
            dy = dy.contiguous()
        dx = torch.empty_like(x, memory_format=torch.contiguous_format)
        need_a = a is not None and ctx.needs_input_grad[1]
        need_c = has_c and ctx.needs_input_grad[2]
        da = torch.zeros(a_shape, dtype=torch.float32, device=x.device) if need_a else None
        dc = torch.zeros(c_shape, dtype=torch.float32, device=x.device) if need_c else None
        ext().ln_mod_bwd(dy, x, mean, rstd, a, a_add, rpg, gidx, rms, dx, None, da, dc, None, None, None, None)
        return dx, da, dc, None, None, None, None, None


def ln_mod(x, a=None, c=None, a_add=1.0, rows_per_group=None, gidx=None, eps=1e-6, rms=False):
    """y = norm(x) * (a_add + a[g]) + c[g] on [R, D] rows; LayerNorm, or RMSNorm if ``rms``."""
    if not x.is_cuda:
        return ln_mod_reference(x, a, c, a_add, rows_per_group, gidx, eps, rms)
    R = x.shape[0]
    rpg = rows_per_group if rows_per_group is not None else max(R, 1)
    a = a.float() if a is not None else None
    c = c.float() if c is not None else None
    gidx = gidx.int().contiguous() if gidx is not None else None
    return _LnMod.apply(x, a, c, a_add, rpg, gidx, eps, rms)


def layer_norm_affine(x, weight, bias, eps=1e-6):
    """Affine LayerNorm over the last dim of [R, D] rows (weight/bias of any float dtype)."""
    return ln_mod(x, weight.reshape(1, -1), bias.reshape(1, -1) if bias is not None else None, a_add=0.0, eps=eps)


def rms_norm(x, weight=None, eps=1e-6):
    """RMSNorm over the last dim of [R, D] rows, optionally scaled by ``weight``."""
    if weight is None:
        return ln_mod(x, None, None, a_add=1.0, eps=eps, rms=True)
    return ln_mod(x, weight.reshape(1, -1), None, a_add=0.0, eps=eps, rms=True)


# ----------------------------------------------------------------------------- gated residual


class _GateRes(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, y, gate, rows_per_group, gidx):
        out = torch.empty_like(x, memory_format=torch.contiguous_format)
        ext().gate_res_fwd(x, y, out, gate, int(rows_per_group), gidx)
        ctx.save_for_backward(y, gate, gidx)
        ctx.rpg = int(rows_per_group)
        return out

    @staticmethod
    def backward(ctx, dout):
        y, gate, gidx = ctx.saved_tensors
        if dout.stride(-1) != 1 or dout.stride(0) % 8:
            dout = dout.contiguous()
        dy = torch.empty_like(y, memory_format=torch.contiguous_format)
        dgate = torch.zeros(gate.shape, dtype=torch.float32, device=y.device)
        ext().gate_res_bwd(dout, y, dy, gate, dgate, ctx.rpg, gidx)
        return dout, dy, (dgate if ctx.needs_input_grad[2] else None), None, None


def gate_residual(x, y, gate=None, rows_per_group=None, gidx=None):
    """x + y * gate[g] on [R, D] rows (gate fp32 [G, D]; None means a plain residual add)."""
    if gate is None:
        return x + y
    if not x.is_cuda:
        R = x.shape[0]
        rpg = rows_per_group if rows_per_group is not None else R
        g = gidx.long() if gidx is not None else torch.arange(R, device=x.device) // max(1, rpg)
        return (x.float() + y.float() * gate.float()[g]).to(x.dtype)
    rpg = rows_per_group if rows_per_group is not None else max(x.shape[0], 1)
    gidx = gidx.int().contiguous() if gidx is not None else None
    return _GateRes.apply(x, y, gate.float(), rpg, gidx)


# ----------------------------------------------------------------------------- RoPE


def rope_reference(x, cos, sin, hd, inverse=False):
    """Interleaved RoPE of [R, H*hd] rows with [Lr, hd/2] tables (row r uses table row r % Lr)."""
    R, D = x.shape
    Lr = cos.shape[0]
    idx = torch.arange(R, device=x.device) % Lr
    c = cos[idx].float()[:, None, :]
    s = sin[idx].float()[:, None, :] * (-1.0 if inverse else 1.0)
    xf = x.float().view(R, D // hd, hd // 2, 2)
    x0, x1 = xf[..., 0], xf[..., 1]
    o0 = x0 * c - x1 * s
    o1 = x1 * c + x0 * s
    return torch.stack([o0, o1], dim=-1).view(R, D).to(x.dtype)


def rope_apply(x, cos, sin, hd=128, inverse=False):
    if not x.is_cuda:
        return rope_reference(x, cos, sin, hd, inverse)
    y = torch.empty_like(x, memory_format=torch.contiguous_format)
    ext().rope_apply(x, y, cos.float().contiguous(), sin.float().contiguous(), int(hd), bool(inverse))
    return y


def qk_norm_rope_reference(src, wq, wk, cos, sin, D, hd, eps):
    q = ln_mod_reference(src[:, :D], wq.reshape(1, -1), None, 0.0, None, None, eps, True)
    k = ln_mod_reference(src[:, D:2 * D], wk.reshape(1, -1), None, 0.0, None, None, eps, True)
    if cos is not None:
        q = rope_reference(q, cos, sin, hd)
        k = rope_reference(k, cos, sin, hd)
    return q, k


def qk_norm_rope(src, wq, wk, cos, sin, D, hd=128, eps=1e-6):
    """(rope(rmsnorm(src[:, :D]) * wq), rope(rmsnorm(src[:, D:2D]) * wk)) as one [R, 2D] buffer.

    Not differentiable on its own: it is the forward half of the attention-core
    autograd functions in ``dmad_b200.models.layers``.
    """
    if not src.is_cuda:
        q, k = qk_norm_rope_reference(src, wq, wk, cos, sin, D, hd, eps)
        return torch.cat([q, k], dim=1), None, None
    R = src.shape[0]
    out = torch.empty((R, 2 * D), dtype=src.dtype, device=src.device)
    rq = torch.empty(R, dtype=torch.float32, device=src.device)
    rk = torch.empty(R, dtype=torch.float32, device=src.device)
    ext().qk_norm_rope_fwd(src, out, wq, wk, cos, sin, rq, rk, int(D), int(hd), float(eps))
    return out, rq, rk


class _Rope(torch.autograd.Function):
    """Differentiable interleaved RoPE: the backward is the inverse rotation."""

    @staticmethod
    def forward(ctx, x, cos, sin, hd):
        ctx.save_for_backward(cos, sin)
        ctx.hd = hd
        y = torch.empty_like(x, memory_format=torch.contiguous_format)
        ext().rope_apply(x, y, cos, sin, int(hd), False)
        return y

    @staticmethod
    def backward(ctx, g):
        cos, sin = ctx.saved_tensors
        g = g.contiguous()
        dx = torch.empty_like(g)
        ext().rope_apply(g, dx, cos, sin, int(ctx.hd), True)
        return dx, None, None, None


def rope(x, cos, sin, hd=128):
    """Differentiable interleaved RoPE of [R, H*hd] rows (row r uses table row r % len(cos))."""
    if not x.is_cuda:
        return rope_reference(x, cos, sin, hd)
    return _Rope.apply(x, cos.float().contiguous(), sin.float().contiguous(), hd)
