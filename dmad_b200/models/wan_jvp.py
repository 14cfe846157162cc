"""Forward-mode JVP of the Wan DiT: (output, d output / d(x, t) . (t_x, t_t)) in one pass.

Parity: train/wan/rcm/networks/wan2pt1_jvp.py:963-1125 (``_forward_jvp``) and the attention JVP of
train/wan/rcm/utils/flash_attention_jvp_triton.py:107-232.  Tangents are propagated op by op:
* Linear: t_y = W t_x (no bias);
* LayerNorm / RMSNorm: t_n = rstd (t_x - mean(t_x) - n mean(n t_x))  (no mean terms for RMS);
* adaLN modulation y = n (1 + s) + c: t_y = t_n (1 + s) + n t_s + t_c;
* gated residual x + y g: t_x + t_y g + y t_g;   GELU: gelu'(x) t_x;   RoPE: the same rotation;
* attention O = softmax(S) V with S = Q K^T * scale:
      t_O = (P (.) t_S) V + P t_V - rowsum(P (.) t_S) O,   t_S = (t_Q K^T + Q t_K^T) * scale;
  cross-attention has no tangent on K, V (the text condition);
* timestep embedding: d/dt [cos(t f), sin(t f)] = [-sin(t f), cos(t f)] f t_t, then the MLP.
The primal of every op is the same kernel as the regular forward.  The attention JVP runs on the
tcgen05 JVP kernel when available and otherwise in blocks of queries with PyTorch matmuls.
"""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F

from .. import ops
from ..ops.norm import rope_reference

_JVP_Q_CHUNK = 2048


def attention_jvp(q, k, v, tq, tk, tv, scale=None):
    """[B, L, H, D] (tk / tv may be None) -> (O, tO) in fp32 math, queries processed in blocks."""
    B, Lq, H, D = q.shape
    scale = scale if scale is not None else 1.0 / math.sqrt(D)
    kf = k.float().transpose(1, 2)
    vf = v.float().transpose(1, 2)
    tkf = tk.float().transpose(1, 2) if tk is not None else None
    tvf = tv.float().transpose(1, 2) if tv is not None else None
    O = torch.empty(B, Lq, H, D, dtype=q.dtype, device=q.device)
    tO = torch.empty_like(O)
    for s in range(0, Lq, _JVP_Q_CHUNK):
        e = min(Lq, s + _JVP_Q_CHUNK)
        qf = q[:, s:e].float().transpose(1, 2)
        tqf = tq[:, s:e].float().transpose(1, 2)
        S = qf @ kf.transpose(-1, -2) * scale
        P = torch.softmax(S, dim=-1)
        del S
        tS = tqf @ kf.transpose(-1, -2)
        if tkf is not None:
            tS = tS + qf @ tkf.transpose(-1, -2)
        tS = tS * scale
        PtS = P * tS
        del tS
        o = P @ vf
        to = PtS @ vf - PtS.sum(-1, keepdim=True) * o
        if tvf is not None:
            to = to + P @ tvf
        O[:, s:e] = o.transpose(1, 2).to(q.dtype)
        tO[:, s:e] = to.transpose(1, 2).to(q.dtype)
    return O, tO


def _attn_jvp(q, k, v, tq, tk, tv):
    if q.is_cuda and ops.native_available() and hasattr(ops.ext(), "flash_jvp_fwd") and q.shape[-1] == 128:
        from ..ops.attention import flash_attention_jvp
        return flash_attention_jvp(q, k, v, tq, tk, tv)
    return attention_jvp(q, k, v, tq, tk, tv)


def _norm_stats(x, rms, eps):
    xf = x.float()
    if rms:
        rstd = torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
        return xf * rstd, rstd
    mu = xf.mean(-1, keepdim=True)
    rstd = torch.rsqrt((xf - mu).pow(2).mean(-1, keepdim=True) + eps)
    return (xf - mu) * rstd, rstd


def _norm_tangent(n, rstd, tx, rms):
    t = tx.float()
    if not rms:
        t = t - t.mean(-1, keepdim=True)
    return rstd * (t - n * (n * tx.float()).mean(-1, keepdim=True))


def _rows(g, rpg, R):
    if torch.is_tensor(rpg):  # explicit group index per row (context-parallel slices)
        return g[rpg.long()]
    return g.repeat_interleave(rpg, dim=0)[:R] if g.shape[0] > 1 else g.expand(R, -1)


def _grp(rpg):
    return {"gidx": rpg} if torch.is_tensor(rpg) else {"rows_per_group": rpg}


def ln_mod_jvp(x, tx, a, ta, c, tc, rpg, eps, a_add=1.0):
    """y = LN(x) (a_add + a) + c with tangent (a / c per group of ``rpg`` rows; ta / tc may be None)."""
    R = x.shape[0]
    y = ops.ln_mod(x, a, c, a_add=a_add, eps=eps, **_grp(rpg))
    n, rstd = _norm_stats(x, False, eps)
    tn = _norm_tangent(n, rstd, tx, False)
    A = a_add + (_rows(a.float(), rpg, R) if a is not None else 0.0)
    ty = tn * A
    if ta is not None:
        ty = ty + n * _rows(ta.float(), rpg, R)
    if tc is not None:
        ty = ty + _rows(tc.float(), rpg, R)
    return y, ty.to(x.dtype)


def rms_jvp(x, tx, w, eps):
    y = ops.rms_norm(x, w, eps)
    n, rstd = _norm_stats(x, True, eps)
    return y, (w.float() * _norm_tangent(n, rstd, tx, True)).to(x.dtype)


def _lin(lin, x, tx):
    w = lin.effective_weight() if hasattr(lin, "effective_weight") else lin.weight
    y = lin(x)
    return y, F.linear(tx.to(w.dtype), w)


def _gate(x, tx, y, ty, g, tg, rpg):
    R = x.shape[0]
    G = _rows(g.float(), rpg, R)
    out = ops.gate_residual(x, y, g, **_grp(rpg))
    t = tx.float() + ty.float() * G + y.float() * _rows(tg.float(), rpg, R)
    return out, t.to(x.dtype)


def _gelu_grad(x):
    k0 = 0.7978845608028654
    x2 = x * x
    u = k0 * (x + 0.044715 * x2 * x)
    th = torch.tanh(u)
    return 0.5 * (1 + th) + 0.5 * x * (1 - th * th) * k0 * (1 + 3 * 0.044715 * x2)


def block_jvp(blk, x, tx, e0, te0, context, cos, sin, B, L, rpg, cp=None, attn_meta=None):
    cfg = blk.cfg
    D, H = cfg.dim, cfg.num_heads
    hd = D // H
    Lc = context.shape[0] // B
    e = blk.modulation.float()[0] + e0
    h, th = ln_mod_jvp(x, tx, e[:, 1], te0[:, 1], e[:, 0], te0[:, 0], rpg, cfg.eps)
    qkv, tqkv = _lin(blk.self_attn.qkv, h, th)
    q, tq = rms_jvp(qkv[:, :D], tqkv[:, :D], blk.self_attn.norm_q.weight, cfg.eps)
    k, tk = rms_jvp(qkv[:, D:2 * D], tqkv[:, D:2 * D], blk.self_attn.norm_k.weight, cfg.eps)
    q, tq = ops.rope_apply(q, cos, sin, hd), ops.rope_apply(tq, cos, sin, hd)
    k, tk = ops.rope_apply(k, cos, sin, hd), ops.rope_apply(tk, cos, sin, hd)
    v, tv = qkv[:, 2 * D:], tqkv[:, 2 * D:]
    if attn_meta is not None and attn_meta.mode != "none":
        from ..ops.block_attention import block_attention_jvp
        shp = (B, L, H, hd)
        a, ta = block_attention_jvp(q.reshape(shp), k.reshape(shp), v.reshape(shp), tq.reshape(shp), tk.reshape(shp),
                                    tv.reshape(shp), attn_meta)
        a, ta = a.reshape(B * L, D), ta.reshape(B * L, D)
    elif cp is not None and cp.world > 1 and cp.impl == "hybrid":
        from ..parallel.cp import hybrid_attention_jvp
        a, ta = hybrid_attention_jvp(q, k, v, tq, tk, tv, B, H, cp)
    elif cp is not None and cp.world > 1 and cp.impl == "ring":
        from ..parallel.cp import ring_attention_jvp
        a, ta = ring_attention_jvp(q, k, v, tq, tk, tv, B, H, cp)
    elif cp is not None and cp.world > 1:
        # the six primal / tangent tensors in one head exchange, the two outputs in one back
        # (the reference's _SeqAllToAllQKVWithT / _SeqAllToAllOutputWithT, jvp_helper.py:69-205)
        g = cp.seq_to_head(torch.cat([q, k, v, tq, tk, tv], dim=1), B, 6, H, hd)
        a, ta = _attn_jvp(g[:, :, 0], g[:, :, 1], g[:, :, 2], g[:, :, 3], g[:, :, 4], g[:, :, 5])
        back = cp.head_to_seq(torch.stack([a, ta], dim=2), B)
        a, ta = back[:, :D], back[:, D:]
    else:
        a, ta = _attn_jvp(q.reshape(B, L, H, hd), k.reshape(B, L, H, hd), v.reshape(B, L, H, hd),
                          tq.reshape(B, L, H, hd), tk.reshape(B, L, H, hd), tv.reshape(B, L, H, hd))
    y, ty = _lin(blk.self_attn.o, a.reshape(B * L, D), ta.reshape(B * L, D))
    x, tx = _gate(x, tx, y, ty, e[:, 2], te0[:, 2], rpg)
    if blk.norm3 is not None:
        h3 = ops.layer_norm_affine(x, blk.norm3.weight, blk.norm3.bias, cfg.eps)
        n3, r3 = _norm_stats(x, False, cfg.eps)
        th3 = (blk.norm3.weight.float() * _norm_tangent(n3, r3, tx, False)).to(x.dtype)
    else:
        h3, th3 = x, tx
    cq, tcq = _lin(blk.cross_attn.q, h3, th3)
    ckv = blk.cross_attn.kv(context)
    cqn, tcqn = rms_jvp(cq, tcq, blk.cross_attn.norm_q.weight, cfg.eps)
    ck = ops.rms_norm(ckv[:, :D], blk.cross_attn.norm_k.weight, cfg.eps)
    c, tc = _attn_jvp(cqn.reshape(B, L, H, hd), ck.reshape(B, Lc, H, hd), ckv[:, D:].reshape(B, Lc, H, hd),
                      tcqn.reshape(B, L, H, hd), None, None)
    co, tco = _lin(blk.cross_attn.o, c.reshape(B * L, D), tc.reshape(B * L, D))
    x, tx = x + co, (tx.float() + tco.float()).to(x.dtype)
    h2, th2 = ln_mod_jvp(x, tx, e[:, 4], te0[:, 4], e[:, 3], te0[:, 3], rpg, cfg.eps)
    f0 = getattr(blk.ffn, "0")
    fpre, tfpre = _lin(f0, h2, th2)
    f = ops.gelu_tanh(fpre)
    tf = (_gelu_grad(fpre.float()) * tfpre.float()).to(fpre.dtype)
    y2, ty2 = _lin(getattr(blk.ffn, "2"), f, tf)
    return _gate(x, tx, y2, ty2, e[:, 5], te0[:, 5], rpg)


def time_embed_jvp(model, t, tt):
    """(e, e0, t_e, t_e0) of the timestep MLP, fp32."""
    D, fd = model.cfg.dim, model.cfg.freq_dim
    half = fd // 2
    freqs = torch.pow(torch.tensor(10000.0, dtype=torch.float64, device=t.device),
                      -torch.arange(half, dtype=torch.float64, device=t.device) / half)
    ph = torch.outer(t.double(), freqs)
    s = torch.cat([torch.cos(ph), torch.sin(ph)], 1).float()
    ts = (torch.cat([-torch.sin(ph), torch.cos(ph)], 1) * freqs.repeat(2)[None] * tt.double()[:, None]).float()
    l0, l2 = model.time_embedding[0], model.time_embedding[2]
    h1 = F.linear(s, l0.weight.float(), l0.bias.float())
    th1 = F.linear(ts, l0.weight.float())
    sg1 = torch.sigmoid(h1)
    a1, ta1 = h1 * sg1, th1 * (sg1 * (1 + h1 * (1 - sg1)))
    e = F.linear(a1, l2.weight.float(), l2.bias.float())
    te = F.linear(ta1, l2.weight.float())
    tp = model.time_projection[1]
    sg2 = torch.sigmoid(e)
    a2, ta2 = e * sg2, te * (sg2 * (1 + e * (1 - sg2)))
    e0 = F.linear(a2, tp.weight.float(), tp.bias.float()).view(-1, 6, D)
    te0 = F.linear(ta2, tp.weight.float()).view(-1, 6, D)
    return e, e0, te, te0


@torch.no_grad()
def wan_forward_jvp(model, x, tx, timesteps, t_timesteps, crossattn_emb, attn_meta=None):
    """(out, t_out) [B, 16, T, H, W] fp32 of ``model`` at (x, timesteps) along (tx, t_timesteps);
    ``attn_meta`` (an ``AttnMaskSpec``) masks the self-attention block-wise (causal modes)."""
    cfg = model.cfg
    if attn_meta is not None and attn_meta.mode != "none" and model.cp is not None and model.cp.world > 1:
        raise NotImplementedError("block masks run without context parallelism")
    cp0 = model.cp if (model.cp is not None and model.cp.world > 1) else None
    if cp0 is not None and cp0.broadcast_inputs:  # rank 0's sample for the whole CP group
        x, tx, crossattn_emb = cp0.broadcast(x), cp0.broadcast(tx), cp0.broadcast(crossattn_emb)
        timesteps, t_timesteps = cp0.broadcast(timesteps), cp0.broadcast(t_timesteps)
    B = x.shape[0]
    wdt = model.patch_embedding.weight.dtype
    xr, (T, H, W) = model.patchify(x.to(wdt))
    txr, _ = model.patchify(tx.to(wdt))
    L = T * H * W
    if timesteps.ndim == 1:
        timesteps, t_timesteps = timesteps[:, None], t_timesteps[:, None]
    uniform = timesteps.shape[1] == 1
    cos, sin = model.rope_tables(T, H, W, xr.device)
    cp = model.cp if (model.cp is not None and model.cp.world > 1) else None
    Ll, r0 = L, 0
    if cp is not None:
        Ll, r0 = L // cp.world, cp.rank * (L // cp.world)
        xr = xr.view(B, L, -1)[:, r0:r0 + Ll].reshape(B * Ll, -1)
        txr = txr.view(B, L, -1)[:, r0:r0 + Ll].reshape(B * Ll, -1)
        cos, sin = cos[r0:r0 + Ll].contiguous(), sin[r0:r0 + Ll].contiguous()
    if uniform:
        rpg = Ll
    elif cp is None:
        rpg = H * W
    else:
        gr = torch.arange(r0, r0 + Ll, device=xr.device) // (H * W)
        rpg = (torch.arange(B, device=xr.device)[:, None] * T + gr[None]).reshape(-1).int()
    h = F.linear(xr, model.patch_embedding.weight, model.patch_embedding.bias)
    th = F.linear(txr, model.patch_embedding.weight)
    e, e0, te, te0 = time_embed_jvp(model, timesteps.reshape(-1).float(), t_timesteps.reshape(-1).float())
    context = model.text_embed(crossattn_emb)
    for blk in model.blocks:
        for hook in blk._forward_pre_hooks.values():  # as blk(...) would: binds sharded block weights
            hook(blk, ())
        h, th = block_jvp(blk, h, th, e0, te0, context, cos, sin, B, Ll, rpg, cp, attn_meta)
    m = model.head.modulation.float()[0]
    ho, tho = ln_mod_jvp(h, th, m[1][None] + e, te, m[0][None] + e, te, rpg, cfg.eps)
    hw = model.head.head
    out = F.linear(ho.float(), hw.weight.float(), hw.bias.float())
    tout = F.linear(tho.float(), hw.weight.float())
    if cp is not None:
        both = cp.gather(torch.cat([out, tout], dim=1).view(B, Ll, -1), dim=1).reshape(B * L, -1)
        out, tout = both[:, :out.shape[1]], both[:, out.shape[1]:]
    return model.unpatchify(out, B, (T, H, W)), model.unpatchify(tout, B, (T, H, W))
