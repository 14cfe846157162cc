"""Block-structured attention masks (block-causal, teacher forcing, local windows, attention sinks).

Parity: train/wan/rcm/utils/blockmask.py:72-389 (``BlockPattern``, ``AttnMaskSpec`` and the mask
predicates of its FlexAttention / Magi paths) -- used by the causal and teacher-forcing modes of the
Wan network; the bidirectional DMAD path never builds a mask.

Every mask of these modes is a union of full rectangles: the queries of one block attend to at most
three contiguous key ranges (sink blocks, the window of earlier blocks ending at the query's block,
and for teacher forcing the query's own noisy block).  So no per-element mask is evaluated: each query
block runs the tcgen05 flash kernel once per key range and the epilogue merges the ranges by their
log-sum-exp (``flash_fwd_accumulate``); the backward runs the flash backward per range with the
merged LSE and adds the partial dK / dV into the range's rows.  The CPU path is the same
decomposition in fp32 PyTorch, and ``dense_mask`` restates the reference's element predicate for
tests.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch

from . import ext


@dataclass(frozen=True)
class BlockPattern:
    """Blocks measured in frames: block 0 has ``first_chunk_frames`` frames, every later block
    ``chunk_frames``; a frame has ``frame_tokens`` tokens."""

    frame_tokens: int = 0
    first_chunk_frames: int = 1
    chunk_frames: int = 1

    def block_frames(self, block: int) -> int:
        return self.first_chunk_frames if block == 0 else self.chunk_frames

    def block_tokens(self, block: int) -> int:
        return self.block_frames(block) * self.frame_tokens

    def blocks_to_frames(self, n: int) -> int:
        return 0 if n <= 0 else self.first_chunk_frames + (n - 1) * self.chunk_frames

    def blocks_to_tokens(self, n: int) -> int:
        return self.blocks_to_frames(n) * self.frame_tokens

    def block_start(self, block: int) -> int:
        """First token of absolute block ``block`` (block 0 is the first chunk)."""
        return self.blocks_to_tokens(block)

    def block_of_token(self, t: int, use_first_block: bool = True) -> int:
        f = t // self.frame_tokens
        if not use_first_block:
            return f // self.chunk_frames
        return 0 if f < self.first_chunk_frames else 1 + (f - self.first_chunk_frames) // self.chunk_frames

    def query_blocks(self, n_tokens: int, block_offset: int = 0):
        """(block, start, end) of the query tokens [0, n_tokens) that begin at absolute block
        ``block_offset`` (the first chunk size applies only when the offset is 0)."""
        out, cur, b = [], 0, block_offset
        while cur < n_tokens:
            n = (self.first_chunk_frames if b == 0 else self.chunk_frames) * self.frame_tokens
            out.append((b, cur, min(n_tokens, cur + n)))
            cur += n
            b += 1
        return out


@dataclass(frozen=True)
class AttnMaskSpec:
    """``mode``: "none" (full attention), "block_causal" (key blocks <= the query's block, full inside a
    block) or "teacher_forcing" (packed [clean][noisy]: clean queries see clean blocks <= theirs, noisy
    queries see earlier clean blocks and their own noisy block).  ``local_attn_blocks`` > 0 keeps only
    the last that many blocks (the current one included); ``sink_blocks`` always admits the first blocks;
    ``q_block_offset`` places the queries after cached blocks; ``clean_blocks`` sizes the clean half."""

    mode: str = "none"
    pattern: BlockPattern | None = None
    local_attn_blocks: int = 0
    sink_blocks: int = 0
    q_block_offset: int = 0
    clean_blocks: int = 0


def _clip(ranges, lo, hi):
    out = []
    for a, b in ranges:
        a, b = max(a, lo), min(b, hi)
        if b > a:
            out.append((a, b))
    return out


def _window(spec: AttnMaskSpec, qb: int, inclusive: bool):
    """(first, last + 1) of the admitted earlier blocks of query block ``qb`` and the sink blocks."""
    last = qb + 1 if inclusive else qb
    lo = max(0, qb - (spec.local_attn_blocks - 1)) if spec.local_attn_blocks > 0 else 0
    sinks = min(spec.sink_blocks, lo, last) if spec.sink_blocks > 0 else 0
    return lo, last, sinks


def mask_ranges(spec: AttnMaskSpec, Q: int, KV: int):
    """[(q0, q1, [(k0, k1), ...])]: the key ranges each query block attends to (rows without any
    admitted key are absent and produce zeros)."""
    if spec.mode == "none":
        return [(0, Q, [(0, KV)])] if Q and KV else []
    pat = spec.pattern
    out = []
    if spec.mode == "block_causal":
        for qb, q0, q1 in pat.query_blocks(Q, spec.q_block_offset):
            lo, last, sinks = _window(spec, qb, inclusive=True)
            rng = [(0, pat.block_start(sinks))] if sinks else []
            rng.append((pat.block_start(lo), pat.block_start(last)))
            rng = _clip(rng, 0, KV)
            if rng:
                out.append((q0, q1, rng))
        return out
    if spec.mode == "teacher_forcing":
        assert spec.clean_blocks > 0, "clean_blocks must be set for teacher_forcing"
        clean = pat.blocks_to_tokens(spec.clean_blocks)
        total = min(2 * clean, Q)
        kv_hi = min(2 * clean, KV)
        for qb, q0, q1 in pat.query_blocks(min(clean, total)):
            lo, last, sinks = _window(spec, qb, inclusive=True)
            rng = ([(0, pat.block_start(sinks))] if sinks else []) + [(pat.block_start(lo), pat.block_start(last))]
            rng = _clip(_clip(rng, 0, clean), 0, kv_hi)
            if rng:
                out.append((q0, q1, rng))
        for qb, q0, q1 in pat.query_blocks(max(0, total - clean)):
            lo, last, sinks = _window(spec, qb, inclusive=False)
            rng = ([(0, pat.block_start(sinks))] if sinks else []) + [(pat.block_start(lo), pat.block_start(last))]
            rng = _clip(rng, 0, clean)
            rng += [(clean + pat.block_start(qb), clean + pat.block_start(qb) + pat.block_tokens(qb))]
            rng = _clip(rng, 0, kv_hi)
            if rng:
                out.append((clean + q0, clean + q1, rng))
        return out
    raise ValueError(f"unknown mask mode {spec.mode!r}")


def dense_mask(spec: AttnMaskSpec, Q: int, KV: int, device=None) -> torch.Tensor:
    """[Q, KV] bool: the element predicate of the reference's mask functions (for tests)."""
    q = torch.arange(Q, device=device)[:, None]
    k = torch.arange(KV, device=device)[None, :]
    if spec.mode == "none":
        return torch.ones(Q, KV, dtype=torch.bool, device=device)
    pat = spec.pattern

    def blk(t, use_first=True):
        f = t // pat.frame_tokens
        if not use_first:
            return f // pat.chunk_frames
        return torch.where(f < pat.first_chunk_frames, torch.zeros_like(f), 1 + (f - pat.first_chunk_frames) //
                           pat.chunk_frames)

    local_k = spec.local_attn_blocks - 1
    if spec.mode == "block_causal":
        qb = spec.q_block_offset + blk(q, spec.q_block_offset == 0)
        kb = blk(k)
        allow = kb <= qb
        if local_k >= 0:
            allow = allow & (kb >= qb - local_k)
        if spec.sink_blocks > 0:
            allow = allow | ((kb < spec.sink_blocks) & (kb <= qb))
        return allow.expand(Q, KV).clone()
    clean = pat.blocks_to_tokens(spec.clean_blocks)
    valid = (q < 2 * clean) & (k < 2 * clean)
    eye = q == k
    qc, kc = q < clean, k < clean
    qbc, qbn, kbc, kbn = blk(q), blk(q - clean), blk(k), blk(k - clean)
    ca = qc & kc & (kbc <= qbc)
    if local_k >= 0:
        ca = ca & (kbc >= qbc - local_k)
    ca = ca | (qc & eye)
    n2c = (~qc) & kc & (kbc < qbn)
    if local_k >= 0:
        n2c = n2c & (kbc >= qbn - local_k)
    na = n2c | ((~qc) & (~kc) & (kbn == qbn)) | ((~qc) & eye)
    if spec.sink_blocks > 0:
        na = na | ((~qc) & kc & (kbc < spec.sink_blocks) & (kbc < qbn))
        ca = ca | (qc & kc & (kbc < spec.sink_blocks) & (kbc < qbc))
    return (valid & (eye | ca | na)).expand(Q, KV).clone()


# ----------------------------------------------------------------------------- attention


def _attn_cpu(q, k, v, blocks, scale):
    ct = torch.promote_types(q.dtype, torch.float32)  # fp32 math (fp64 inputs stay fp64)
    out = torch.zeros(q.shape, dtype=ct, device=q.device)
    for q0, q1, rng in blocks:
        kk = torch.cat([k[:, a:b] for a, b in rng], dim=1).to(ct).transpose(1, 2)
        vv = torch.cat([v[:, a:b] for a, b in rng], dim=1).to(ct).transpose(1, 2)
        s = q[:, q0:q1].to(ct).transpose(1, 2) @ kk.transpose(-1, -2) * scale
        o = torch.softmax(s, -1) @ vv
        out = out.index_copy(1, torch.arange(q0, q1, device=q.device), o.transpose(1, 2))
    return out.to(q.dtype)


def _lse_pad(n):
    return (n + 255) // 256 * 256


class _BlockAttn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, blocks, scale):
        e = ext()
        B, Q, H, D = q.shape
        o = torch.zeros_like(q, memory_format=torch.contiguous_format)
        lses = []
        for q0, q1, rng in blocks:
            qs, os_ = q[:, q0:q1], o[:, q0:q1]
            lse = torch.empty((B, H, _lse_pad(q1 - q0)), dtype=torch.float32, device=q.device)
            if len(rng) == 1:
                a, b = rng[0]
                e.flash_fwd(qs, k[:, a:b], v[:, a:b], os_, lse, float(scale))
            else:
                acc_o = torch.empty((B, q1 - q0, H, D), dtype=torch.float32, device=q.device)
                acc_lse = torch.empty_like(lse)
                for j, (a, b) in enumerate(rng):
                    e.flash_fwd_accumulate(qs, k[:, a:b], v[:, a:b], os_, lse, acc_o, acc_lse, j > 0,
                                           j == len(rng) - 1, float(scale))
            lses.append(lse)
        ctx.save_for_backward(q, k, v, o, *lses)
        ctx.blocks, ctx.scale = blocks, scale
        return o

    @staticmethod
    def backward(ctx, do):
        from .attention import flash_bwd_into

        q, k, v, o, *lses = ctx.saved_tensors
        do = do.contiguous()
        dq = torch.zeros(q.shape, dtype=torch.float32, device=q.device)
        dk = torch.zeros(k.shape, dtype=torch.float32, device=q.device)
        dv = torch.zeros(v.shape, dtype=torch.float32, device=q.device)
        for (q0, q1, rng), lse in zip(ctx.blocks, lses):
            qs, os_, dos = q[:, q0:q1], o[:, q0:q1], do[:, q0:q1]
            dd = torch.empty_like(lse)
            for a, b in rng:
                gq, gk, gv = torch.empty_like(qs), torch.empty_like(k[:, a:b]), torch.empty_like(v[:, a:b])
                flash_bwd_into(qs, k[:, a:b], v[:, a:b], os_, dos, lse, gq, gk, gv, dd, ctx.scale)
                dq[:, q0:q1] += gq.float()
                dk[:, a:b] += gk.float()
                dv[:, a:b] += gv.float()
        return dq.to(q.dtype), dk.to(k.dtype), dv.to(v.dtype), None, None


def block_attention(q, k, v, spec: AttnMaskSpec | None = None, scale: float | None = None):
    """softmax(q k^T scale + mask) v for [B, Q, H, D] queries and [B, KV, H, D] keys / values under a
    block mask (``None`` or mode "none" = full attention)."""
    spec = spec or AttnMaskSpec()
    scale = float(scale) if scale is not None else 1.0 / math.sqrt(q.shape[-1])
    blocks = mask_ranges(spec, q.shape[1], k.shape[1])
    if not q.is_cuda:
        return _attn_cpu(q, k, v, blocks, scale)
    return _BlockAttn.apply(q, k, v, blocks, scale)


# ----------------------------------------------------------------------------- JVP under a block mask


def _jvp_cpu(q, k, v, tq, tk, tv, blocks, scale):
    ct = torch.promote_types(q.dtype, torch.float32)
    O = torch.zeros(q.shape, dtype=ct, device=q.device)
    tO = torch.zeros(q.shape, dtype=ct, device=q.device)
    hv = lambda t: t.to(ct).transpose(1, 2)  # noqa: E731
    for q0, q1, rng in blocks:
        cat = lambda t: hv(torch.cat([t[:, a:b] for a, b in rng], dim=1))  # noqa: E731
        kk, vv = cat(k), cat(v)
        qq, tqq = hv(q[:, q0:q1]), hv(tq[:, q0:q1])
        s = qq @ kk.transpose(-1, -2) * scale
        ts = tqq @ kk.transpose(-1, -2)
        if tk is not None:
            ts = ts + qq @ cat(tk).transpose(-1, -2)
        p = torch.softmax(s, -1)
        pts = p * (ts * scale)
        o = p @ vv
        to = pts @ vv - pts.sum(-1, keepdim=True) * o
        if tv is not None:
            to = to + p @ cat(tv)
        O[:, q0:q1] = o.transpose(1, 2)
        tO[:, q0:q1] = to.transpose(1, 2)
    return O.to(q.dtype), tO.to(q.dtype)


@torch.no_grad()
def block_attention_jvp(q, k, v, tq, tk=None, tv=None, spec: AttnMaskSpec | None = None, scale: float | None = None):
    """(O, tO): attention under a block mask and its forward-mode derivative along (tq, tk, tv) (None =
    zero tangent), [B, L, H, D].  Forward only; on CUDA one tcgen05 JVP launch per key range with the
    ranges merged by (LSE, mu = rowsum(P * tS) / l) in the epilogue (``flash_jvp_accumulate``).
    Parity: the reference's masked Triton JVP (flash_attention_jvp_triton.py:235-409)."""
    spec = spec or AttnMaskSpec()
    scale = float(scale) if scale is not None else 1.0 / math.sqrt(q.shape[-1])
    blocks = mask_ranges(spec, q.shape[1], k.shape[1])
    if not q.is_cuda:
        return _jvp_cpu(q, k, v, tq, tk, tv, blocks, scale)
    e = ext()
    B, Q, H, D = q.shape
    q, tq = q.contiguous(), tq.contiguous()
    o, to = torch.zeros_like(q), torch.zeros_like(q)
    no_lse = torch.empty(0, dtype=torch.float32, device=q.device)
    sl = lambda t, a, b: t[:, a:b].contiguous() if t is not None else None  # noqa: E731
    for q0, q1, rng in blocks:
        qs, tqs, os_, tos = q[:, q0:q1], tq[:, q0:q1], o[:, q0:q1], to[:, q0:q1]
        if len(rng) == 1:
            a, b = rng[0]
            e.flash_jvp_fwd(qs, k[:, a:b], v[:, a:b], tqs, sl(tk, a, b), sl(tv, a, b), os_, tos, no_lse, scale)
            continue
        n = q1 - q0
        acc_o = torch.empty((B, n, H, D), dtype=torch.float32, device=q.device)
        acc_u = torch.empty_like(acc_o)
        acc_lse = torch.empty((B, H, _lse_pad(n)), dtype=torch.float32, device=q.device)
        acc_mu = torch.empty_like(acc_lse)
        for j, (a, b) in enumerate(rng):
            e.flash_jvp_accumulate(qs, k[:, a:b], v[:, a:b], tqs, sl(tk, a, b), sl(tv, a, b), os_, tos, no_lse,
                                   acc_o, acc_u, acc_lse, acc_mu, j > 0, j == len(rng) - 1, scale)
    return o, to
