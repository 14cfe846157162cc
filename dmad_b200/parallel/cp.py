"""Ulysses context parallelism (sequence sharding with a head all-to-all around attention).

Every rank of a context-parallel (CP) group holds the contiguous token slice
``[r*Ll, (r+1)*Ll)`` of every sample (``Ll = L / cp``).  Everything but self-attention is
row-local.  Self-attention exchanges sequence shards for head shards (each rank then attends
over the full sequence with ``H / cp`` heads) and back.  Parity: the reference's
``DistributedAttention`` / ``_SeqAllToAllQKV`` / ``_SeqAllToAll``
(train/wan/rcm/utils/a2a_cp.py:43-258), ``split_inputs_cp`` / ``cat_outputs_cp(_with_grad)``
(train/wan/rcm/utils/context_parallel.py:25-210) and the CP handling of ``WanModel.forward``
(train/wan/rcm/networks/wan2pt1.py:723-823).

Two implementations of the exchange, selected by ``impl``:

* ``"fused"`` -- this framework's kernels over NVLink peer memory.  The q/k RMSNorm + RoPE
  kernel stores q, k and v straight into the head-sharded receive slot of the rank that owns
  each head; the flash-attention epilogue stores each output row into its owner's row buffer
  as well as locally; the backward uses plain peer-copy kernels.  Each exchange ends with the
  bounded-wait ``PeerSync`` barrier.  Receive slots come from one symmetric arena with two
  slots used alternately by successive exchanges: a rank pushes into slot s again only after
  the barrier of the exchange in between, which every peer enters after the kernels that read
  slot s (stream order), so no push overwrites data that is still being read.
* ``"nccl"`` -- ``all_to_all_single`` on permuted copies, as the reference does (the baseline).

On CPU (gloo ranks, tests) only ``"nccl"`` is available and attention runs in fp32 PyTorch.
"""
from __future__ import annotations

import math

import torch
import torch.distributed as dist

from .dist import is_distributed
from .symm import PeerSync, SymmBuffer


class ContextParallel:
    def __init__(self, group=None, impl: str = "fused", device=None, timeout_s: float = 120.0,
                 broadcast_inputs: bool = True):
        if impl not in ("fused", "nccl", "ring"):
            raise ValueError(f"unknown context-parallel impl {impl!r}")
        self.group = group if group is not None else (dist.group.WORLD if is_distributed() else None)
        self.world = dist.get_world_size(self.group) if self.group is not None else 1
        self.rank = dist.get_rank(self.group) if self.group is not None else 0
        self.device = torch.device(device) if device is not None else (
            torch.device("cuda", torch.cuda.current_device()) if torch.cuda.is_available() else torch.device("cpu"))
        if self.device.type != "cuda" and impl == "fused":
            impl = "nccl"
        self.impl = impl
        self.timeout_s = timeout_s
        self.broadcast_inputs = broadcast_inputs
        self._arena: SymmBuffer | None = None
        self._slot_elems = 0
        self._op = 0
        self.sync = PeerSync(self.device, self.group, timeout_s) if impl in ("fused", "ring") and \
            self.device.type == "cuda" else None
        self.ring_stream = torch.cuda.Stream(device=self.device) if impl == "ring" and self.device.type == "cuda" \
            else None
        self._ring_bufs = None

    # ------------------------------------------------------------------ symmetric receive slots
    def reserve(self, elems: int):
        """Make both slots hold at least ``elems`` bf16 elements (collective; same value on all ranks)."""
        elems = -(-elems // 64) * 64
        if elems <= self._slot_elems:
            return
        if self._arena is not None:
            torch.cuda.synchronize(self.device)
        self._arena = SymmBuffer(2 * elems, torch.bfloat16, self.device, self.group, zero=False)
        self._slot_elems = elems

    def slot(self, elems: int):
        """(local view [elems], peer addresses) of the next slot."""
        self.reserve(elems)
        s = self._op & 1
        self._op += 1
        base = s * self._slot_elems
        view = self._arena.tensor[base:base + elems]
        ptrs = [p + base * 2 for p in self._arena.ptrs]
        return view, ptrs

    def ring_buffers(self, elems: int):
        """Two local bf16 buffers for the key/value blocks copied from peers (ring attention)."""
        if self._ring_bufs is None or self._ring_bufs[0].numel() < elems:
            self._ring_bufs = [torch.empty(elems, dtype=torch.bfloat16, device=self.device) for _ in range(2)]
        return self._ring_bufs

    # ------------------------------------------------------------------ token sharding (cold path)
    def split(self, x: torch.Tensor, dim: int = 1) -> torch.Tensor:
        n = x.shape[dim]
        assert n % self.world == 0, f"sequence length {n} must be divisible by cp={self.world}"
        ll = n // self.world
        return x.narrow(dim, self.rank * ll, ll).contiguous()

    def gather(self, x: torch.Tensor, dim: int = 1) -> torch.Tensor:
        """all_gather along ``dim``; differentiable (each rank keeps the gradient of its own slice)."""
        if self.world == 1:
            return x
        return _GatherSeq.apply(x, dim, self)

    def all_reduce_sum(self, t: torch.Tensor) -> torch.Tensor:
        """Sum over the CP group; the gradient passes through unchanged (each rank's local term)."""
        if self.world == 1:
            return t
        return _AllReduceSum.apply(t, self)

    def broadcast(self, t: torch.Tensor, src_rank_in_group: int = 0) -> torch.Tensor:
        """Values of the group's rank ``src_rank_in_group``; the gradient flows to the local input
        unchanged (context_parallel.py:167-190 ``item + (bcast - item.detach())``)."""
        if self.world == 1:
            return t
        return _Broadcast.apply(t, src_rank_in_group, self)

    # ------------------------------------------------------------------ exchanges (either implementation)
    def seq_to_head(self, rows: torch.Tensor, B: int, n: int, H: int, hd: int) -> torch.Tensor:
        """[B*Ll, n*H*hd] local rows -> [B, L, n, Hl, hd] head shard of the full sequence.  The fused
        result is a view of a receive slot: consume it before two more exchanges (or clone it)."""
        if self.impl == "nccl" or not rows.is_cuda:
            return self.a2a_seq_to_head(rows, B, n, H, hd)
        from .. import ops
        from ..runtime.nvtx import nvtx_range

        Hl = H // self.world
        L = rows.shape[0] // B * self.world
        slot, ptrs = self.slot(B * L * n * Hl * hd)
        rows = rows if (rows.stride(-1) == 1 and rows.stride(0) % 8 == 0) else rows.contiguous()
        with nvtx_range("dmad.cp.seq_to_head"):
            ops.ext().cp_seq_to_head(rows, ptrs, B, H * hd, n, hd, self.rank)
            self.sync()
        return slot.view(B, L, n, Hl, hd)

    def head_to_seq(self, y: torch.Tensor, B: int) -> torch.Tensor:
        """[B, L, n, Hl, hd] -> [B*Ll, n*H*hd] local rows (a slot view when fused)."""
        if self.impl == "nccl" or not y.is_cuda:
            return self.a2a_head_to_seq(y.contiguous(), B, y.shape[2])
        from .. import ops

        _, L, n, Hl, hd = y.shape
        D = Hl * self.world * hd
        R = B * (L // self.world)
        slot, ptrs = self.slot(R * n * D)
        ops.ext().cp_head_to_seq([y[:, :, i] for i in range(n)], ptrs, n * D, D, self.rank)
        self.sync()
        return slot.view(R, n * D)

    # ------------------------------------------------------------------ NCCL all-to-all (baseline)
    def a2a_seq_to_head(self, x: torch.Tensor, B: int, n: int, H: int, hd: int) -> torch.Tensor:
        """[B*Ll, n*H*hd] rows -> [B, L, n, Hl, hd] (NCCL)."""
        cp, Hl = self.world, H // self.world
        Ll = x.shape[0] // B
        send = x.reshape(B, Ll, n, cp, Hl, hd).permute(3, 0, 1, 2, 4, 5).contiguous()
        recv = torch.empty_like(send)
        dist.all_to_all_single(recv, send, group=self.group)
        return recv.permute(1, 0, 2, 3, 4, 5).reshape(B, cp * Ll, n, Hl, hd)

    def a2a_head_to_seq(self, y: torch.Tensor, B: int, n: int) -> torch.Tensor:
        """[B, L, n, Hl, hd] -> [B*Ll, n*H*hd] rows (NCCL)."""
        cp = self.world
        _, L, _, Hl, hd = y.shape
        Ll = L // cp
        send = y.reshape(B, cp, Ll, n, Hl, hd).permute(1, 0, 2, 3, 4, 5).contiguous()
        recv = torch.empty_like(send)
        dist.all_to_all_single(recv, send, group=self.group)
        # recv[src] = rows of my slice, heads of rank src
        return recv.permute(1, 2, 3, 0, 4, 5).reshape(B * Ll, n * cp * Hl * hd)


class _GatherSeq(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, dim, cp):
        ctx.dim, ctx.cp = dim, cp
        parts = [torch.empty_like(x) for _ in range(cp.world)]
        dist.all_gather(parts, x.contiguous(), group=cp.group)
        return torch.cat(parts, dim=dim)

    @staticmethod
    def backward(ctx, g):
        cp = ctx.cp
        ll = g.shape[ctx.dim] // cp.world
        return g.narrow(ctx.dim, cp.rank * ll, ll).contiguous(), None, None


class _GatherSum(torch.autograd.Function):
    """All-gather along ``dim`` whose consumers differ per rank (attention over gathered keys): the
    backward sums every rank's gradient of a slice and returns this rank's slice (reduce-scatter)."""

    @staticmethod
    def forward(ctx, x, dim, cp):
        parts = [torch.empty_like(x) for _ in range(cp.world)]
        dist.all_gather(parts, x.contiguous(), group=cp.group)
        ctx.cfg = (dim, cp, x.shape[dim])
        return torch.cat(parts, dim=dim)

    @staticmethod
    def backward(ctx, g):
        dim, cp, n = ctx.cfg
        g = g.contiguous()
        dist.all_reduce(g, group=cp.group)
        return g.narrow(dim, cp.rank * n, n).contiguous(), None, None


class _Broadcast(torch.autograd.Function):
    @staticmethod
    def forward(ctx, t, src_in_group, cp):
        out = t.detach().clone().contiguous()
        src = dist.get_global_rank(cp.group, src_in_group) if cp.group is not dist.group.WORLD else src_in_group
        dist.broadcast(out, src=src, group=cp.group)
        return out

    @staticmethod
    def backward(ctx, g):
        return g, None, None


class _AllReduceSum(torch.autograd.Function):
    @staticmethod
    def forward(ctx, t, cp):
        t = t.clone()
        dist.all_reduce(t, group=cp.group)
        return t

    @staticmethod
    def backward(ctx, g):
        return g, None


# ---------------------------------------------------------------------- self-attention under CP
class _SelfAttnCP(torch.autograd.Function):
    """qkv [B*Ll, 3D] (pre-norm, local rows) -> attention output [B*Ll, D] over the full sequence.

    cos / sin: RoPE tables of this rank's Ll rows."""

    @staticmethod
    def forward(ctx, qkv, wq, wk, cos, sin, B, H, eps, cp):
        from .. import ops
        from ..ops import attention as attn_ops
        from ..ops import norm as norm_ops

        e = ops.ext()
        R, D3 = qkv.shape
        D = D3 // 3
        hd = D // H
        Hl = H // cp.world
        Ll = R // B
        L = Ll * cp.world
        scale = 1.0 / math.sqrt(hd)
        if cp.impl == "fused":
            slot, ptrs = cp.slot(B * L * 3 * Hl * hd)
            rq = torch.empty(R, dtype=torch.float32, device=qkv.device)
            rk = torch.empty_like(rq)
            e.cp_qkv_push(qkv, ptrs, wq, wk, cos, sin, rq, rk, B, D, hd, cp.rank, eps)
            cp.sync()
            qkv_g = slot.view(B, L, 3, Hl, hd)
            if any(ctx.needs_input_grad):
                qkv_g = qkv_g.clone()  # kept for backward; the slot is reused two exchanges later
        else:
            qk, rq, rk = norm_ops.qk_norm_rope(qkv, wq, wk, cos, sin, D, hd, eps)
            rows = torch.cat([qk, qkv[:, 2 * D:]], dim=1)
            qkv_g = cp.a2a_seq_to_head(rows, B, 3, H, hd)
        q_g, k_g, v_g = qkv_g[:, :, 0], qkv_g[:, :, 1], qkv_g[:, :, 2]
        o_g = torch.empty((B, L, Hl, hd), dtype=qkv.dtype, device=qkv.device)
        lse = torch.empty((B, Hl, attn_ops._lse_pad(L)), dtype=torch.float32, device=qkv.device)
        if cp.impl == "fused":
            oslot, optrs = cp.slot(R * D)
            e.flash_fwd_scatter(q_g, k_g, v_g, o_g, lse, scale, optrs, D, cp.rank * Hl * hd)
            cp.sync()
            out = oslot.view(R, D).clone()
        else:
            e.flash_fwd(q_g, k_g, v_g, o_g, lse, scale)
            out = cp.a2a_head_to_seq(o_g.view(B, L, 1, Hl, hd), B, 1)
        ctx.save_for_backward(qkv, wq, wk, cos, sin, rq, rk, qkv_g, o_g, lse)
        ctx.cfg = (B, H, eps, scale, cp)
        return out

    @staticmethod
    def backward(ctx, do):
        from .. import ops
        from ..ops import attention as attn_ops

        qkv, wq, wk, cos, sin, rq, rk, qkv_g, o_g, lse = ctx.saved_tensors
        B, H, eps, scale, cp = ctx.cfg
        e = ops.ext()
        R, D3 = qkv.shape
        D = D3 // 3
        hd = D // H
        Hl = H // cp.world
        Ll = R // B
        L = Ll * cp.world
        do = do.contiguous()
        if cp.impl == "fused":
            dslot, dptrs = cp.slot(B * L * Hl * hd)
            e.cp_seq_to_head(do, dptrs, B, D, 1, hd, cp.rank)
            cp.sync()
            do_g = dslot.view(B, L, Hl, hd)
        else:
            do_g = cp.a2a_seq_to_head(do, B, 1, H, hd)[:, :, 0]
        dqkv_g = torch.empty((B, L, 3, Hl, hd), dtype=qkv.dtype, device=qkv.device)
        dd = torch.empty_like(lse)
        attn_ops.flash_bwd_into(qkv_g[:, :, 0], qkv_g[:, :, 1], qkv_g[:, :, 2], o_g, do_g, lse, dqkv_g[:, :, 0],
                    dqkv_g[:, :, 1], dqkv_g[:, :, 2], dd, scale)
        if cp.impl == "fused":
            gslot, gptrs = cp.slot(R * 3 * D)
            e.cp_head_to_seq([dqkv_g[:, :, 0], dqkv_g[:, :, 1], dqkv_g[:, :, 2]], gptrs, 3 * D, D, cp.rank)
            cp.sync()
            g_rows = gslot.view(R, 3 * D)
        else:
            g_rows = cp.a2a_head_to_seq(dqkv_g, B, 3)
        dqkv = torch.empty_like(qkv)
        dqkv[:, 2 * D:].copy_(g_rows[:, 2 * D:])
        dwq = torch.zeros(D, dtype=torch.float32, device=qkv.device)
        dwk = torch.zeros(D, dtype=torch.float32, device=qkv.device)
        e.qk_norm_rope_bwd(g_rows[:, :D], g_rows[:, D:2 * D], qkv, dqkv, wq, wk, cos, sin, rq, rk, dwq, dwk, D, hd)
        return dqkv, dwq, dwk, None, None, None, None, None, None


def self_attention_cp(qkv, wq, wk, cos, sin, B, H, eps, cp: ContextParallel):
    """Self-attention of the local rows ``qkv`` [B*Ll, 3D] against the whole CP-sharded sequence."""
    if not qkv.is_cuda:
        return _self_attention_cp_cpu(qkv, wq, wk, cos, sin, B, H, eps, cp)
    return _SelfAttnCP.apply(qkv, wq.float().contiguous(), wk.float().contiguous(), cos, sin, B, H, eps, cp)


def _self_attention_cp_cpu(qkv, wq, wk, cos, sin, B, H, eps, cp):
    """fp32 PyTorch path (gloo ranks): the same exchange through differentiable all-to-alls."""
    from ..ops import attention as attn_ops
    from ..ops import norm as norm_ops

    R, D3 = qkv.shape
    D = D3 // 3
    hd = D // H
    q = norm_ops.ln_mod_reference(qkv[:, :D], wq.reshape(1, -1), None, 0.0, None, None, eps, True)
    k = norm_ops.ln_mod_reference(qkv[:, D:2 * D], wk.reshape(1, -1), None, 0.0, None, None, eps, True)
    q = norm_ops.rope_reference(q, cos, sin, hd)
    k = norm_ops.rope_reference(k, cos, sin, hd)
    rows = torch.cat([q, k, qkv[:, 2 * D:]], dim=1)
    g = _A2ASeqToHead.apply(rows, B, 3, H, hd, cp)
    o = attn_ops.attention_reference(g[:, :, 0], g[:, :, 1], g[:, :, 2])
    return _A2AHeadToSeq.apply(o.unsqueeze(2), B, 1, H, cp)


class _A2ASeqToHead(torch.autograd.Function):
    @staticmethod
    def forward(ctx, rows, B, n, H, hd, cp):
        ctx.cfg = (B, n, H, cp)
        return cp.a2a_seq_to_head(rows, B, n, H, hd)

    @staticmethod
    def backward(ctx, g):
        B, n, H, cp = ctx.cfg
        return cp.a2a_head_to_seq(g.contiguous(), B, n), None, None, None, None, None


class _A2AHeadToSeq(torch.autograd.Function):
    @staticmethod
    def forward(ctx, y, B, n, H, cp):
        ctx.cfg = (B, n, H, y.shape[-1], cp)
        return cp.a2a_head_to_seq(y.contiguous(), B, n)

    @staticmethod
    def backward(ctx, g):
        B, n, H, hd, cp = ctx.cfg
        return cp.a2a_seq_to_head(g.contiguous(), B, n, H, hd), None, None, None, None


# ---------------------------------------------------------------------- ring attention
# impl="ring": every rank keeps the queries of its own tokens (all heads) and visits the key / value
# block of every rank.  Each rank's normalised k and v sit in a symmetric slot; the block of the next
# rank is copied into a local double buffer by the copy engine on a side stream while the flash kernel
# works on the current block, and the kernel's epilogue merges the block into an fp32 running output
# with its log-sum-exp (flash_fwd_accumulate).  The backward visits the blocks again with the final
# LSE: dQ accumulates locally, the dK / dV partials of a block are pushed into per-source slots of
# its owner and summed there.  Parity: there is no ring attention in the reference (Ulysses only,
# train/wan/rcm/utils/a2a_cp.py); this is the ring variant of the same context parallelism.

def _ring_blocks(cp, slot_ptrs, nbytes, stream, bufs, visit):
    """Call ``visit(j, src, kv)`` for the key/value block (``nbytes`` of each rank's slot) of every rank
    ``src = rank + j`` (``kv`` None for this rank's own block).  The block of step j + 1 is copied into
    ``bufs[(j + 1) % 2]`` on ``stream`` while step j computes; a copy starts only after the work that
    last read its buffer."""
    from .. import ops

    e = ops.ext()
    cur = torch.cuda.current_stream()
    ready = {}

    def prefetch(j):
        src = (cp.rank + j) % cp.world
        ev = torch.cuda.Event()
        ev.record(cur)
        with torch.cuda.stream(stream):
            stream.wait_event(ev)
            e.peer_copy(bufs[j & 1], slot_ptrs[src], nbytes)
            done = torch.cuda.Event()
            done.record(stream)
        ready[j] = done

    if cp.world > 1:
        prefetch(1)
    for j in range(cp.world):
        if 1 <= j < cp.world - 1:
            prefetch(j + 1)  # its buffer was last read by step j - 1, already issued
        kv = None
        if j > 0:
            cur.wait_event(ready[j])
            kv = bufs[j & 1]
        visit(j, (cp.rank + j) % cp.world, kv)
    cur.wait_stream(stream)


class _RingSelfAttn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, qkv, wq, wk, cos, sin, B, H, eps, cp):
        from .. import ops
        from ..ops import attention as attn_ops
        from ..ops import norm as norm_ops

        e = ops.ext()
        R, D3 = qkv.shape
        D = D3 // 3
        hd = D // H
        Ll = R // B
        scale = 1.0 / math.sqrt(hd)
        qk, rq, rk = norm_ops.qk_norm_rope(qkv, wq, wk, cos, sin, D, hd, eps)
        q = qk[:, :D].view(B, Ll, H, hd)
        slot, ptrs = cp.slot(2 * R * D)
        own = slot.view(2, R, D)
        own[0].copy_(qk[:, D:])
        own[1].copy_(qkv[:, 2 * D:])
        cp.sync()  # every rank's block is in place
        o = torch.empty((B, Ll, H, hd), dtype=qkv.dtype, device=qkv.device)
        lse = torch.empty((B, H, attn_ops._lse_pad(Ll)), dtype=torch.float32, device=qkv.device)
        acc_o = torch.empty((B, Ll, H, hd), dtype=torch.float32, device=qkv.device)
        acc_lse = torch.empty_like(lse)
        bufs = cp.ring_buffers(2 * R * D)

        def visit(j, src, kv):
            blk = own if kv is None else kv.view(2, R, D)
            e.flash_fwd_accumulate(q, blk[0].view(B, Ll, H, hd), blk[1].view(B, Ll, H, hd), o, lse, acc_o, acc_lse,
                                   j > 0, j == cp.world - 1, scale)

        _ring_blocks(cp, ptrs, 2 * R * D * 2, cp.ring_stream, bufs, visit)
        cp.sync()  # the peers have copied this rank's block before the slot is reused
        ctx.save_for_backward(qkv, wq, wk, cos, sin, rq, rk, o, lse)
        ctx.cfg = (B, H, eps, scale, cp)
        return o.view(R, D)

    @staticmethod
    def backward(ctx, do):
        from .. import ops
        from ..ops import attention as attn_ops
        from ..ops import norm as norm_ops

        qkv, wq, wk, cos, sin, rq, rk, o, lse = ctx.saved_tensors
        B, H, eps, scale, cp = ctx.cfg
        e = ops.ext()
        R, D3 = qkv.shape
        D = D3 // 3
        hd = D // H
        Ll = R // B
        qk, _, _ = norm_ops.qk_norm_rope(qkv, wq, wk, cos, sin, D, hd, eps)
        q = qk[:, :D].view(B, Ll, H, hd)
        slot, ptrs = cp.slot(2 * R * D)
        own = slot.view(2, R, D)
        own[0].copy_(qk[:, D:])
        own[1].copy_(qkv[:, 2 * D:])
        part, pptrs = cp.slot(cp.world * 2 * R * D)  # [source rank, dK | dV, R, D] of this rank's block
        cp.sync()
        do = do.contiguous().view(B, Ll, H, hd)
        dq_acc = torch.zeros((R, D), dtype=torch.float32, device=qkv.device)
        dq = torch.empty((B, Ll, H, hd), dtype=qkv.dtype, device=qkv.device)
        dkv = torch.empty((2, R, D), dtype=qkv.dtype, device=qkv.device)
        dd = torch.empty_like(lse)
        bufs = cp.ring_buffers(2 * R * D)
        part_v = part.view(cp.world, 2, R, D)

        def visit(j, src, kv):
            blk = own if kv is None else kv.view(2, R, D)
            attn_ops.flash_bwd_into(q, blk[0].view(B, Ll, H, hd), blk[1].view(B, Ll, H, hd), o, do, lse, dq,
                        dkv[0].view(B, Ll, H, hd), dkv[1].view(B, Ll, H, hd), dd, scale)
            dq_acc.add_(dq.view(R, D).float())
            if src == cp.rank:
                part_v[cp.rank].copy_(dkv)
            else:  # into the owner's slot for this source rank (copy engine)
                e.peer_copy_to(pptrs[src] + cp.rank * 2 * R * D * 2, dkv, 2 * R * D * 2)
            # dkv is reused by the next block: wait for the copy (same stream, ordered)

        _ring_blocks(cp, ptrs, 2 * R * D * 2, cp.ring_stream, bufs, visit)
        cp.sync()  # every partial has landed
        g = part_v.float().sum(0)
        dqk = torch.cat([dq_acc, g[0]], dim=1).to(qkv.dtype)
        dqkv = torch.empty_like(qkv)
        dqkv[:, 2 * D:].copy_(g[1].to(qkv.dtype))
        dwq = torch.zeros(D, dtype=torch.float32, device=qkv.device)
        dwk = torch.zeros(D, dtype=torch.float32, device=qkv.device)
        e.qk_norm_rope_bwd(dqk[:, :D], dqk[:, D:], qkv, dqkv, wq, wk, cos, sin, rq, rk, dwq, dwk, D, hd)
        return dqkv, dwq, dwk, None, None, None, None, None, None


def _ring_cpu(qkv, wq, wk, cos, sin, B, H, eps, cp):
    """fp32 restatement of ring attention (gloo ranks): all-gather the blocks, merge per block by LSE."""
    from ..ops import norm as norm_ops

    R, D3 = qkv.shape
    D = D3 // 3
    hd = D // H
    Ll = R // B
    q = norm_ops.rope_reference(norm_ops.ln_mod_reference(qkv[:, :D], wq.reshape(1, -1), None, 0.0, None, None, eps,
                                                          True), cos, sin, hd)
    k = norm_ops.rope_reference(norm_ops.ln_mod_reference(qkv[:, D:2 * D], wk.reshape(1, -1), None, 0.0, None, None,
                                                          eps, True), cos, sin, hd)
    kv = torch.cat([k, qkv[:, 2 * D:]], dim=1)
    blocks = _GatherSum.apply(kv.view(1, R, 2 * D), 1, cp).view(cp.world, R, 2 * D)
    qf = q.float().view(B, Ll, H, hd).transpose(1, 2)
    acc, lse = None, None
    for j in range(cp.world):
        src = (cp.rank + j) % cp.world
        kj = blocks[src, :, :D].float().view(B, Ll, H, hd).transpose(1, 2)
        vj = blocks[src, :, D:].float().view(B, Ll, H, hd).transpose(1, 2)
        s = qf @ kj.transpose(-1, -2) / math.sqrt(hd)
        l_j = torch.logsumexp(s, -1, keepdim=True)
        o_j = torch.softmax(s, -1) @ vj
        if acc is None:
            acc, lse = o_j, l_j
        else:
            nl = torch.logaddexp(lse, l_j)
            acc = acc * torch.exp(lse - nl) + o_j * torch.exp(l_j - nl)
            lse = nl
    return acc.transpose(1, 2).reshape(R, D).to(qkv.dtype)


def ring_self_attention(qkv, wq, wk, cos, sin, B, H, eps, cp: ContextParallel):
    if not qkv.is_cuda:
        return _ring_cpu(qkv, wq, wk, cos, sin, B, H, eps, cp)
    return _RingSelfAttn.apply(qkv, wq.float().contiguous(), wk.float().contiguous(), cos, sin, B, H, eps, cp)


# ---------------------------------------------------------------------- ring attention JVP
# The tangent pass of the student (sCM / rCM targets) on the ring: each rank's slot holds k, v, tk,
# tv of its tokens; every block is merged by flash_jvp_accumulate, whose epilogue keeps O, T~/l, the
# log-sum-exp and mu = rowsum(P * tS) / l of the blocks seen so far and writes tO = T~/l - mu O at the
# last block.  Runs without autograd, as every JVP of the DMAD objectives does.  Parity: the Ulysses
# form of the same exchange is the reference's _SeqAllToAllQKVWithT (train/wan/rcm/utils/
# jvp_helper.py:69-205); the ring form is this build's.

def ring_attention_jvp(q, k, v, tq, tk, tv, B: int, H: int, cp: ContextParallel):
    """Local rows [R, D] of q, k, v and their tangents -> (O, tO) rows [R, D] of attention over the
    sequence of the whole CP group (this rank's queries, every rank's keys)."""
    if torch.is_grad_enabled() and any(t.requires_grad for t in (q, k, v)):
        raise RuntimeError("ring_attention_jvp is forward-only: call it under torch.no_grad()")
    if not q.is_cuda:
        return _ring_jvp_cpu(q, k, v, tq, tk, tv, B, H, cp)
    from .. import ops
    from ..ops import attention as attn_ops

    e = ops.ext()
    R, D = q.shape
    hd = D // H
    Ll = R // B
    scale = 1.0 / math.sqrt(hd)
    slot, ptrs = cp.slot(4 * R * D)
    own = slot.view(4, R, D)
    for i, t in enumerate((k, v, tk, tv)):
        own[i].copy_(t)
    cp.sync()  # every rank's block is in place
    shp = (B, Ll, H, hd)
    q4, tq4 = q.contiguous().view(shp), tq.contiguous().view(shp)
    o = torch.empty(shp, dtype=q.dtype, device=q.device)
    to = torch.empty_like(o)
    acc_o = torch.empty(shp, dtype=torch.float32, device=q.device)
    acc_u = torch.empty_like(acc_o)
    acc_lse = torch.empty((B, H, attn_ops._lse_pad(Ll)), dtype=torch.float32, device=q.device)
    acc_mu = torch.empty_like(acc_lse)
    no_lse = torch.empty(0, dtype=torch.float32, device=q.device)
    bufs = cp.ring_buffers(4 * R * D)

    def visit(j, src, kv):
        blk = own if kv is None else kv[:4 * R * D].view(4, R, D)
        e.flash_jvp_accumulate(q4, blk[0].view(shp), blk[1].view(shp), tq4, blk[2].view(shp), blk[3].view(shp),
                               o, to, no_lse, acc_o, acc_u, acc_lse, acc_mu, j > 0, j == cp.world - 1, scale)

    _ring_blocks(cp, ptrs, 4 * R * D * 2, cp.ring_stream, bufs, visit)
    cp.sync()  # the peers have copied this rank's block before the slot is reused
    return o.view(R, D), to.view(R, D)


def _ring_jvp_cpu(q, k, v, tq, tk, tv, B, H, cp):
    """fp32 restatement (gloo ranks): gather the blocks, merge (O, T~/l, mu) per block by LSE."""
    R, D = q.shape
    hd = D // H
    Ll = R // B
    blocks = cp.gather(torch.cat([k, v, tk, tv], dim=1).view(1, R, 4 * D), dim=1).view(cp.world, R, 4 * D)
    hv = lambda t: t.float().reshape(B, Ll, H, hd).transpose(1, 2)  # noqa: E731
    qf, tqf = hv(q), hv(tq)
    scale = 1.0 / math.sqrt(hd)
    O = U = mu = lse = None
    for j in range(cp.world):
        blk = blocks[(cp.rank + j) % cp.world]
        kj, vj, tkj, tvj = (hv(blk[:, i * D:(i + 1) * D]) for i in range(4))
        s = qf @ kj.transpose(-1, -2) * scale
        ts = (tqf @ kj.transpose(-1, -2) + qf @ tkj.transpose(-1, -2)) * scale
        l_j = torch.logsumexp(s, -1, keepdim=True)
        p = torch.exp(s - l_j)
        o_j = p @ vj
        u_j = p @ tvj + (p * ts) @ vj
        mu_j = (p * ts).sum(-1, keepdim=True)
        if O is None:
            O, U, mu, lse = o_j, u_j, mu_j, l_j
        else:
            nl = torch.logaddexp(lse, l_j)
            wa, wb = torch.exp(lse - nl), torch.exp(l_j - nl)
            O, U, mu, lse = O * wa + o_j * wb, U * wa + u_j * wb, mu * wa + mu_j * wb, nl
    tO = U - mu * O
    back = lambda t: t.transpose(1, 2).reshape(R, D).to(q.dtype)  # noqa: E731
    return back(O), back(tO)


# ---------------------------------------------------------------------- hybrid: Ulysses inside, ring across
# For head counts the CP size does not divide (H3's 40 heads at cp = 16, for instance) the group of
# cp = u * r ranks is split into r Ulysses groups of u consecutive ranks and u ring groups of r ranks
# with the same position.  A Ulysses group exchanges heads for sequence inside itself, so each rank
# holds its group's whole span of L / r tokens for H / u heads; the ring then visits the spans of the
# other groups for the same heads (key/value blocks through the copy engine, LSE merge in the flash
# epilogue), and the Ulysses exchange runs back.  Parity: the reference has Ulysses only
# (train/wan/rcm/utils/a2a_cp.py); the hybrid is this build's extension of it.

class HybridContextParallel:
    """``ContextParallel``-compatible group of ``u * r`` ranks: ``.ulysses`` (u consecutive ranks) and
    ``.ring`` (r ranks with the same Ulysses position), each a ``ContextParallel``."""

    impl = "hybrid"

    def __init__(self, group=None, ulysses_size: int = 2, device=None, timeout_s: float = 120.0,
                 ulysses_impl: str = "fused", broadcast_inputs: bool = True):
        self.full = ContextParallel(group, impl="nccl", device=device, timeout_s=timeout_s,
                                    broadcast_inputs=broadcast_inputs)
        self.group, self.world, self.rank = self.full.group, self.full.world, self.full.rank
        self.device, self.broadcast_inputs, self.timeout_s = self.full.device, broadcast_inputs, timeout_s
        u = int(ulysses_size)
        if u < 1 or self.world % u:
            raise ValueError(f"ulysses_size {u} must divide the CP size {self.world}")
        ranks = dist.get_process_group_ranks(self.group) if self.group is not None else list(range(self.world))
        r = self.world // u
        # only the members of a sub-group create it (so CP groups of different data-parallel replicas
        # need not make the same calls)
        i, j = self.rank // u, self.rank % u
        mine_u = dist.new_group(ranks[i * u:(i + 1) * u], use_local_synchronization=True)
        mine_r = dist.new_group(ranks[j::u], use_local_synchronization=True)
        self.ulysses = ContextParallel(mine_u, impl=ulysses_impl, device=device, timeout_s=timeout_s,
                                       broadcast_inputs=False)
        self.ring = ContextParallel(mine_r, impl="ring", device=device, timeout_s=timeout_s, broadcast_inputs=False)
        self.u, self.r = u, r

    # whole-group helpers (token sharding, broadcasts, reductions) delegate to the full group
    def split(self, x, dim=1):
        return self.full.split(x, dim)

    def gather(self, x, dim=1):
        return self.full.gather(x, dim)

    def all_reduce_sum(self, t):
        return self.full.all_reduce_sum(t)

    def broadcast(self, t, src_rank_in_group: int = 0):
        return self.full.broadcast(t, src_rank_in_group)


def _ring_core_fwd(q, kv_rows, cp: ContextParallel, valid: int | None = None):
    """q [B, Lr, Hl, hd]; kv_rows [2, B*Lr, Hl*hd] (k, v of this rank's span) -> (o, lse) over the spans
    of every rank of the ring group; ``valid`` (B = 1) = the global number of real keys, so the padded
    tail of the last spans is left out."""
    from .. import ops
    from ..ops import attention as attn_ops

    e = ops.ext()
    B, Lr, Hl, hd = q.shape
    R, D = B * Lr, Hl * hd
    scale = 1.0 / math.sqrt(hd)
    slot, ptrs = cp.slot(2 * R * D)
    own = slot.view(2, R, D)
    own.copy_(kv_rows)
    cp.sync()
    o = torch.empty((B, Lr, Hl, hd), dtype=q.dtype, device=q.device)
    lse = torch.empty((B, Hl, attn_ops._lse_pad(Lr)), dtype=torch.float32, device=q.device)
    acc_o = torch.empty((B, Lr, Hl, hd), dtype=torch.float32, device=q.device)
    acc_lse = torch.empty_like(lse)
    bufs = cp.ring_buffers(2 * R * D)
    shp = (B, Lr, Hl, hd)
    nkeys = [Lr if valid is None else max(0, min(Lr, valid - ((cp.rank + j) % cp.world) * Lr))
             for j in range(cp.world)]
    last = max((j for j in range(cp.world) if nkeys[j] > 0), default=-1)
    first = min((j for j in range(cp.world) if nkeys[j] > 0), default=-1)

    def visit(j, src, kv):
        n = nkeys[j]
        if n == 0:
            return
        blk = own if kv is None else kv[:2 * R * D].view(2, R, D)
        e.flash_fwd_accumulate(q, blk[0].view(shp)[:, :n], blk[1].view(shp)[:, :n], o, lse, acc_o, acc_lse,
                               j > first, j == last, scale)

    _ring_blocks(cp, ptrs, 2 * R * D * 2, cp.ring_stream, bufs, visit)
    cp.sync()
    if last < 0:
        o.zero_()
    return o, lse


def _ring_core_bwd(q, kv_rows, o, lse, do, cp: ContextParallel):
    """(dq [B, Lr, Hl, hd], dkv [2, B*Lr, Hl*hd]) of the ring attention of ``_ring_core_fwd``."""
    from .. import ops
    from ..ops import attention as attn_ops

    e = ops.ext()
    B, Lr, Hl, hd = q.shape
    R, D = B * Lr, Hl * hd
    scale = 1.0 / math.sqrt(hd)
    shp = (B, Lr, Hl, hd)
    slot, ptrs = cp.slot(2 * R * D)
    own = slot.view(2, R, D)
    own.copy_(kv_rows)
    part, pptrs = cp.slot(cp.world * 2 * R * D)
    cp.sync()
    dq_acc = torch.zeros((B, Lr, Hl, hd), dtype=torch.float32, device=q.device)
    dq = torch.empty(shp, dtype=q.dtype, device=q.device)
    dkv = torch.empty((2, R, D), dtype=q.dtype, device=q.device)
    dd = torch.empty_like(lse)
    bufs = cp.ring_buffers(2 * R * D)
    part_v = part.view(cp.world, 2, R, D)

    def visit(j, src, kv):
        blk = own if kv is None else kv[:2 * R * D].view(2, R, D)
        attn_ops.flash_bwd_into(q, blk[0].view(shp), blk[1].view(shp), o, do, lse, dq, dkv[0].view(shp),
                                dkv[1].view(shp), dd, scale)
        dq_acc.add_(dq.float())
        if src == cp.rank:
            part_v[cp.rank].copy_(dkv)
        else:
            e.peer_copy_to(pptrs[src] + cp.rank * 2 * R * D * 2, dkv, 2 * R * D * 2)

    _ring_blocks(cp, ptrs, 2 * R * D * 2, cp.ring_stream, bufs, visit)
    cp.sync()
    return dq_acc.to(q.dtype), part_v.float().sum(0).to(q.dtype)


class _HybridSelfAttn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, qkv, wq, wk, cos, sin, B, H, eps, hcp):
        from ..ops import norm as norm_ops

        R, D3 = qkv.shape
        D = D3 // 3
        hd = D // H
        u = hcp.ulysses
        qk, rq, rk = norm_ops.qk_norm_rope(qkv, wq, wk, cos, sin, D, hd, eps)
        g = u.seq_to_head(torch.cat([qk, qkv[:, 2 * D:]], dim=1), B, 3, H, hd)  # [B, Lr, 3, Hl, hd]
        q_h = g[:, :, 0].contiguous()
        kv_rows = g[:, :, 1:].permute(2, 0, 1, 3, 4).reshape(2, -1, (H // u.world) * hd)
        o_h, lse = _ring_core_fwd(q_h, kv_rows, hcp.ring)
        out = u.head_to_seq(o_h.unsqueeze(2), B).clone()
        ctx.save_for_backward(qkv, wq, wk, cos, sin, rq, rk, q_h, kv_rows, o_h, lse)
        ctx.cfg = (B, H, eps, hcp)
        return out

    @staticmethod
    def backward(ctx, do):
        from .. import ops

        qkv, wq, wk, cos, sin, rq, rk, q_h, kv_rows, o_h, lse = ctx.saved_tensors
        B, H, eps, hcp = ctx.cfg
        u = hcp.ulysses
        R, D3 = qkv.shape
        D = D3 // 3
        hd = D // H
        do_h = u.seq_to_head(do.contiguous(), B, 1, H, hd)[:, :, 0].contiguous()
        dq_h, dkv = _ring_core_bwd(q_h, kv_rows, o_h, lse, do_h, hcp.ring)
        Bq, Lr, Hl, _ = q_h.shape
        grads = torch.stack([dq_h, dkv[0].view(Bq, Lr, Hl, hd), dkv[1].view(Bq, Lr, Hl, hd)], dim=2)
        back = u.head_to_seq(grads, B)  # [R, 3D]: dq | dk | dv rows
        dqkv = torch.empty_like(qkv)
        dqkv[:, 2 * D:].copy_(back[:, 2 * D:])
        dwq = torch.zeros(D, dtype=torch.float32, device=qkv.device)
        dwk = torch.zeros(D, dtype=torch.float32, device=qkv.device)
        dqk = back[:, :2 * D].contiguous()
        ops.ext().qk_norm_rope_bwd(dqk[:, :D], dqk[:, D:], qkv, dqkv, wq, wk, cos, sin, rq, rk, dwq, dwk, D, hd)
        return dqkv, dwq, dwk, None, None, None, None, None, None


def _hybrid_cpu(qkv, wq, wk, cos, sin, B, H, eps, hcp):
    """fp32 restatement on gloo ranks: Ulysses exchange (NCCL-style all-to-all), all-gather of the ring
    group's keys / values, attention, exchange back (differentiable end to end)."""
    from ..ops import attention as attn_ops
    from ..ops import norm as norm_ops

    R, D3 = qkv.shape
    D = D3 // 3
    hd = D // H
    q, k = norm_ops.qk_norm_rope_reference(qkv, wq, wk, cos, sin, D, hd, eps)
    u = hcp.ulysses
    g = _A2ASeqToHead.apply(torch.cat([q, k, qkv[:, 2 * D:]], dim=1), B, 3, H, hd, u)  # [B, Lr, 3, Hl, hd]
    kv = _GatherSum.apply(g[:, :, 1:].contiguous(), 1, hcp.ring)  # [B, L, 2, Hl, hd]
    o = attn_ops.attention_reference(g[:, :, 0], kv[:, :, 0], kv[:, :, 1])
    return _A2AHeadToSeq.apply(o.unsqueeze(2).contiguous(), B, 1, H, u)


def hybrid_self_attention(qkv, wq, wk, cos, sin, B, H, eps, hcp: HybridContextParallel):
    if not qkv.is_cuda:
        return _hybrid_cpu(qkv, wq, wk, cos, sin, B, H, eps, hcp)
    return _HybridSelfAttn.apply(qkv, wq.float().contiguous(), wk.float().contiguous(), cos, sin, B, H, eps, hcp)


@torch.no_grad()
def hybrid_attention_fwd(q, k, v, B: int, H: int, hcp: HybridContextParallel, valid: int | None = None):
    """Forward-only hybrid attention of normalised / rotated rows ([B*Ll, D] each) -> [B*Ll, D];
    ``valid`` leaves the padded tail of the global sequence out of every softmax (B = 1)."""
    from ..ops import attention as attn_ops

    R, D = q.shape
    hd = D // H
    u = hcp.ulysses
    g = u.seq_to_head(torch.cat([q, k, v], dim=1), B, 3, H, hd)  # [B, Lr, 3, Hl, hd]
    if not q.is_cuda:
        kv = hcp.ring.gather(g[:, :, 1:].contiguous(), dim=1)
        n = kv.shape[1] if valid is None else valid
        o = attn_ops.attention_reference(g[:, :, 0], kv[:, :n, 0], kv[:, :n, 1])
        return u.head_to_seq(o.unsqueeze(2).contiguous(), B)
    q_h = g[:, :, 0].contiguous()
    kv_rows = g[:, :, 1:].permute(2, 0, 1, 3, 4).reshape(2, -1, (H // u.world) * hd)
    o_h, _ = _ring_core_fwd(q_h, kv_rows, hcp.ring, valid)
    return u.head_to_seq(o_h.unsqueeze(2), B).clone()


@torch.no_grad()
def hybrid_attention_jvp(q, k, v, tq, tk, tv, B: int, H: int, hcp: HybridContextParallel):
    """(O, tO) rows of the hybrid attention (Ulysses exchange of the six tensors, ring JVP, exchange back)."""
    R, D = q.shape
    hd = D // H
    u = hcp.ulysses
    Hl = H // u.world
    g = u.seq_to_head(torch.cat([q, k, v, tq, tk, tv], dim=1), B, 6, H, hd)  # [B, Lr, 6, Hl, hd]
    rows = [g[:, :, i].reshape(-1, Hl * hd).contiguous() for i in range(6)]
    o, to = ring_attention_jvp(*rows, B, Hl, hcp.ring)
    Lr = rows[0].shape[0] // B
    back = u.head_to_seq(torch.stack([o.view(B, Lr, Hl, hd), to.view(B, Lr, Hl, hd)], dim=2).contiguous(), B)
    return back[:, :D].clone(), back[:, D:].clone()


def make_context_parallel(group=None, impl: str = "fused", device=None, ulysses_size: int | None = None,
                          timeout_s: float = 120.0):
    """``ContextParallel`` (impl fused / nccl / ring) or ``HybridContextParallel`` (impl "hybrid":
    Ulysses groups of ``ulysses_size`` ranks, ring across them)."""
    if impl == "hybrid":
        return HybridContextParallel(group, ulysses_size or 2, device=device, timeout_s=timeout_s)
    return ContextParallel(group, impl=impl, device=device, timeout_s=timeout_s)
