"""Sharded data-parallel AdamW: reduce-scatter, update and all-gather in one kernel.

Every trainable parameter of a group lives in one flat symmetric buffer (``p.data`` is a
view into it) and its gradient in a second one (``p.grad`` is a view; autograd accumulates
into it in place).  Rank r owns the shard ``[r * len, (r + 1) * len)`` of the flat vector
and holds the fp32 master weights, Adam moments and (optionally) the EMA of that shard
only, so optimiser state costs 12-16 bytes per parameter / world size.

One optimiser step on the GPU is

    PeerSync()                      every rank's backward is done (gradients complete)
    [dp_sumsq; PeerSync(payload)]   only when clipping: global norm from per-shard partials
    dp_adamw                        pull peer gradients of my shard (or one NVLS multicast
                                    load that the switch sums), AdamW on my fp32 shard, push the
                                    new bf16 weights into every rank's parameter buffer
                                    (or one NVLS multicast store)
    PeerSync()                      every rank has its new weights; gradients may be zeroed

which replaces the NCCL all-reduce of the gradients plus a replicated optimiser step.
Parity target: FSDP2 ``fully_shard`` + FusedAdam(master_weights=True)
(train/wan/rcm/models/t2v_model_distill_rcm.py:175-195,
train/wan/rcm/utils/fused_adam_dtensor.py:29-416).

Without CUDA (CPU tests on gloo ranks) the same algorithm runs on torch collectives: the
flat gradient is all-reduced, each rank updates its shard and the shards are all-gathered.
"""
from __future__ import annotations

import math
from typing import Iterable

import torch
import torch.distributed as dist

from .dist import get_rank, get_world_size, is_distributed
from .symm import PeerSync, SymmBuffer

_ALIGN = 8  # elements; every parameter view starts on a 16-byte boundary (bf16)


class _FlatGroup:
    def __init__(self, params, dtype, device, world, rank, group, want_ema, sync_timeout_s):
        self.params = params
        self.dtype = dtype
        self.offsets = []
        n = 0
        for p in params:
            self.offsets.append(n)
            n += -(-p.numel() // _ALIGN) * _ALIGN
        self.numel = n
        gran = _ALIGN * 8
        self.len = max(gran, -(-n // (world * gran)) * gran)  # shard length (elements)
        self.total = self.len * world
        self.off = rank * self.len
        self.pbuf = SymmBuffer(self.total, dtype, device, group)
        self.gbuf = SymmBuffer(self.total, dtype, device, group)
        with torch.no_grad():
            for p, o in zip(params, self.offsets):
                view = self.pbuf.tensor[o:o + p.numel()].view_as(p)
                view.copy_(p.data)
                p.data = view
                p.grad = self.gbuf.tensor[o:o + p.numel()].view_as(p)
        shard = self.pbuf.tensor[self.off:self.off + self.len]
        self.master = shard.float().clone()
        self.exp_avg = torch.zeros_like(self.master)
        self.exp_avg_sq = torch.zeros_like(self.master)
        self.ema = self.master.clone() if want_ema else None
        self.mc = self.pbuf.mc_ptr != 0 and self.gbuf.mc_ptr != 0

    def grad_views(self):
        for p, o in zip(self.params, self.offsets):
            yield p, self.gbuf.tensor[o:o + p.numel()].view_as(p)


class ShardedAdamW:
    """AdamW over flat symmetric buffers, one fused reduce-scatter/update/all-gather per step.

    ``ema=True`` keeps an fp32 EMA of the shard, advanced in the same kernel
    (``step(ema_beta=...)``).  ``use_multicast`` selects the NVLS path when the fabric offers it.
    """

    def __init__(self, params: Iterable[torch.nn.Parameter], lr=1e-4, betas=(0.9, 0.999), eps=1e-8,
                 weight_decay=0.0, ema: bool = False, group=None, use_multicast: bool = True,
                 sync_timeout_s: float = 120.0, force_finite: bool = False):
        self.force_finite = force_finite
        self.params = [p for p in params]
        self.lr, self.betas, self.eps, self.weight_decay = lr, tuple(betas), eps, weight_decay
        self.step_count = 0
        self.group = group
        self.world = get_world_size(group)
        self.rank = get_rank() if group is None else dist.get_rank(group)
        dev = self.params[0].device
        self.device = dev
        by_dtype: dict = {}
        for p in self.params:
            by_dtype.setdefault(p.dtype, []).append(p)
        self.groups = [_FlatGroup(ps, dt, dev, self.world, self.rank, group, ema, sync_timeout_s)
                       for dt, ps in sorted(by_dtype.items(), key=lambda kv: str(kv[0]))]
        self.use_multicast = use_multicast
        self.sync = PeerSync(dev, group, sync_timeout_s)
        self._acc = torch.zeros(1, dtype=torch.float32, device=dev)
        self.has_ema = ema

    @property
    def param_groups(self):
        return [{"params": self.params, "lr": self.lr}]

    @property
    def multicast(self) -> bool:
        return self.use_multicast and all(g.mc for g in self.groups)

    def zero_grad(self, set_to_none: bool = True):
        """Zero the flat gradient buffers (the per-parameter views stay attached)."""
        for g in self.groups:
            g.gbuf.tensor.zero_()
            for p, view in g.grad_views():
                if p.grad is None or p.grad.data_ptr() != view.data_ptr():
                    p.grad = view

    def _check_views(self):
        for g in self.groups:
            for p, view in g.grad_views():
                if p.grad is None:
                    p.grad = view
                elif p.grad.data_ptr() != view.data_ptr():
                    # autograd replaced the view (e.g. the user set grads to None): fold it back in
                    view.copy_(p.grad)
                    p.grad = view

    @torch.no_grad()
    def step(self, grad_scale: torch.Tensor | None = None, ema_beta: float | None = None,
             max_grad_norm: float | None = None):
        if grad_scale is not None:
            raise ValueError("ShardedAdamW computes the clipping scale itself: pass max_grad_norm")
        self.step_count += 1
        self._check_views()
        clip = max_grad_norm is not None and not math.isinf(max_grad_norm) and max_grad_norm < 1e11
        if self.device.type != "cuda":
            self._step_host(ema_beta, max_grad_norm if clip else None)
            return
        from ..ops import ext
        from ..runtime.nvtx import nvtx_range

        with nvtx_range("dmad.dp_step"):
            self._step_device(ext, ema_beta, max_grad_norm, clip)

    def _step_device(self, ext, ema_beta, max_grad_norm, clip):
        b1, b2 = self.betas
        mc = self.multicast
        self.sync()
        slots = None
        if clip:
            self._acc.zero_()
            for g in self.groups:
                ext().dp_sumsq(g.gbuf.ptrs, g.pbuf.ptrs, g.gbuf.mc_ptr if mc else 0, g.pbuf.mc_ptr if mc else 0,
                               g.pbuf.tensor.element_size(), g.off, g.len, self._acc, self.force_finite)
            self.sync(self._acc)
            slots = self.sync.slots
        for g in self.groups:
            ext().dp_adamw(g.gbuf.ptrs, g.pbuf.ptrs, g.gbuf.mc_ptr if mc else 0, g.pbuf.mc_ptr if mc else 0,
                           g.pbuf.tensor.element_size(), g.master, g.exp_avg, g.exp_avg_sq,
                           g.ema if ema_beta is not None else None, g.off, g.len, float(self.lr), float(b1),
                           float(b2), float(self.eps), float(self.weight_decay), int(self.step_count),
                           float(ema_beta) if ema_beta is not None else 0.0, slots,
                           float(max_grad_norm) if clip else 0.0, self.force_finite)
        self.sync()

    # ------------------------------------------------------------------ host path (gloo / CPU)
    def _step_host(self, ema_beta, max_norm):
        b1, b2 = self.betas
        bc1 = 1 - b1 ** self.step_count
        bc2 = 1 - b2 ** self.step_count
        dist_on = is_distributed() and self.world > 1
        shards = []
        for g in self.groups:
            flat = g.gbuf.tensor.float()
            if dist_on:
                dist.all_reduce(flat, group=self.group)
            sh = flat[g.off:g.off + g.len] / self.world
            if self.force_finite:
                sh = torch.nan_to_num(sh, nan=0.0, posinf=0.0, neginf=0.0)
            shards.append(sh)
        scale = 1.0
        if max_norm is not None:
            ss = torch.stack([(s * s).sum() for s in shards]).sum().reshape(1)
            if dist_on:
                dist.all_reduce(ss, group=self.group)
            n = float(ss.sqrt())
            scale = min(1.0, max_norm / (n + 1e-6)) if math.isfinite(n) else 0.0
        for g, gs in zip(self.groups, shards):
            gs = gs * scale
            w = g.master
            w.mul_(1 - self.lr * self.weight_decay)
            g.exp_avg.mul_(b1).add_(gs, alpha=1 - b1)
            g.exp_avg_sq.mul_(b2).addcmul_(gs, gs, value=1 - b2)
            denom = (g.exp_avg_sq / bc2).sqrt_().add_(self.eps)
            w.addcdiv_(g.exp_avg, denom, value=-self.lr / bc1)
            if g.ema is not None and ema_beta is not None:
                g.ema.mul_(ema_beta).add_(w, alpha=1 - ema_beta)
            new = w.to(g.dtype)
            if dist_on:
                parts = [torch.empty_like(new) for _ in range(self.world)]
                dist.all_gather(parts, new, group=self.group)
                g.pbuf.tensor.copy_(torch.cat(parts))
            else:
                g.pbuf.tensor[g.off:g.off + g.len].copy_(new)

    # ------------------------------------------------------------------ full views (checkpoint / export)
    def _gather(self, shard_of) -> list[torch.Tensor]:
        out = []
        for g in self.groups:
            shard = shard_of(g)
            if is_distributed() and self.world > 1:
                parts = [torch.empty_like(shard) for _ in range(self.world)]
                dist.all_gather(parts, shard.contiguous(), group=self.group)
                full = torch.cat(parts)
            else:
                full = shard
            for p, o in zip(g.params, g.offsets):
                out.append((p, full[o:o + p.numel()].view(p.shape)))
        order = {id(p): i for i, p in enumerate(self.params)}
        out.sort(key=lambda t: order[id(t[0])])
        return [t for _, t in out]

    def full_master(self) -> list[torch.Tensor]:
        return self._gather(lambda g: g.master)

    def full_ema(self) -> list[torch.Tensor] | None:
        if not self.has_ema:
            return None
        return self._gather(lambda g: g.ema)

    def layout(self, names: dict | None = None) -> list[dict]:
        """Flat-buffer layout of every group: shard length, world and (name, offset, shape) per parameter
        (``names``: id(param) -> name), so full tensors can be rebuilt from the per-rank shards offline."""
        out = []
        for g in self.groups:
            out.append({"dtype": str(g.dtype), "len": g.len, "world": self.world,
                        "params": [((names or {}).get(id(p), str(i)), o, tuple(p.shape))
                                   for i, (p, o) in enumerate(zip(g.params, g.offsets))]})
        return out

    def state_dict(self):
        """This rank's shard state (save one file per rank, or gather with ``full_*``)."""
        return {"step": self.step_count, "lr": self.lr, "world": self.world, "rank": self.rank,
                "shards": [{"off": g.off, "len": g.len, "master": g.master, "exp_avg": g.exp_avg,
                            "exp_avg_sq": g.exp_avg_sq, "ema": g.ema} for g in self.groups]}

    def load_resharded(self, rank_states: list[dict]):
        """Elastic resume: load the shard states of every rank of a run with another world size (the flat
        parameter layout is the same; only the shard boundaries move)."""
        states = sorted(rank_states, key=lambda r: r["rank"])
        if len(states) != int(states[0]["world"]):
            raise ValueError(f"need the states of all {states[0]['world']} ranks, got {len(states)}")
        self.step_count = int(states[0]["step"])
        self.lr = states[0].get("lr", self.lr)
        for gi, g in enumerate(self.groups):
            for key in ("master", "exp_avg", "exp_avg_sq", "ema"):
                dst = getattr(g, key)
                parts = [st["shards"][gi].get(key) for st in states]
                if dst is None or any(p is None for p in parts):
                    continue
                dst.copy_(reshard_flat(parts, g.total, g.off, g.len).to(dst.device, dst.dtype))
            new = g.master.to(g.dtype)
            if is_distributed() and self.world > 1:
                parts = [torch.empty_like(new) for _ in range(self.world)]
                dist.all_gather(parts, new, group=self.group)
                g.pbuf.tensor.copy_(torch.cat(parts))
            else:
                g.pbuf.tensor[g.off:g.off + g.len].copy_(new)

    def load_state_dict(self, sd):
        if int(sd["world"]) != self.world:
            raise ValueError(f"sharded state was saved with world {sd['world']}, running with {self.world}")
        self.step_count = int(sd["step"])
        self.lr = sd.get("lr", self.lr)
        for g, s in zip(self.groups, sd["shards"]):
            g.master.copy_(s["master"])
            g.exp_avg.copy_(s["exp_avg"])
            g.exp_avg_sq.copy_(s["exp_avg_sq"])
            if g.ema is not None and s.get("ema") is not None:
                g.ema.copy_(s["ema"])
            new = g.master.to(g.dtype)
            if is_distributed() and self.world > 1:
                parts = [torch.empty_like(new) for _ in range(self.world)]
                dist.all_gather(parts, new, group=self.group)
                g.pbuf.tensor.copy_(torch.cat(parts))
            else:
                g.pbuf.tensor[g.off:g.off + g.len].copy_(new)


def reshard_flat(parts: list[torch.Tensor], total: int, off: int, length: int) -> torch.Tensor:
    """This rank's ``[off, off + length)`` slice of the flat buffer that the old ranks' shards ``parts``
    (in rank order) tile; the old and new flat lengths may differ only in the zero padding at the end."""
    full = torch.cat([p.float().reshape(-1) for p in parts])
    if full.numel() < total:
        full = torch.cat([full, full.new_zeros(total - full.numel())])
    return full[off:off + length].clone()


def tensors_from_shards(layout: list[dict], rank_states: list[dict], key: str = "ema") -> dict:
    """Rebuild full fp32 tensors (name -> tensor) from every rank's ``state_dict()`` shards
    (``key``: "master", "ema", "exp_avg" or "exp_avg_sq"), e.g. to export the EMA offline."""
    out = {}
    for gi, g in enumerate(layout):
        parts = [rs["shards"][gi][key] for rs in sorted(rank_states, key=lambda r: r["rank"])]
        if any(p is None for p in parts):
            raise KeyError(f"shard state {key!r} missing")
        full = torch.cat([p.float().cpu() for p in parts])
        for name, off, shape in g["params"]:
            n = 1
            for d in shape:
                n *= d
            out[name] = full[off:off + n].view(shape).clone()
    return out
