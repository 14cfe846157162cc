"""FSDP-style sharding of the frozen weights of a block stack, gathered one block ahead.

The frozen bf16 weights of every block (the LoRA student's base, the teacher, H3's 33B blocks)
are flattened per block and split over the group: rank r keeps the shard
``[r * len, (r + 1) * len)`` in a symmetric buffer and frees the full tensors.  A forward
pre-hook on block i binds the block's parameters to a gathered copy in one of three rotating
local slots, and a peer-pull kernel on a side stream (csrc/fsdp.cu) gathers the next block in the
direction of travel (i + 1 in forward, i - 1 in the backward recomputation) while block i runs.
The side stream waits for an event recorded at block i's pre-hook before it overwrites a slot, and
the compute stream waits for the gather of a block before using it.  Shards are written once, so
no barrier is needed per gather.

Blocks sharded this way must be activation-checkpointed when they run with grad: autograd would
otherwise keep views of a slot that a later gather overwrites (``check_checkpointing`` asserts it).
Parity: FSDP2 ``fully_shard`` per block with ``reshard_after_forward`` (train/wan/rcm/models/
t2v_model_distill_rcm.py:175-195, train/wan/rcm/networks/wan2pt1.py:882-888,
train/h3/lightx2v_train/runtime/fsdp.py:60-85); there the all-gather is NCCL, here it is a
peer-memory copy overlapped with the previous block's compute.
"""
from __future__ import annotations

import torch
import torch.distributed as dist
import torch.nn as nn

from .dist import barrier, get_rank, get_world_size, is_distributed
from .symm import SymmBuffer

_ALIGN = 8


class ShardedFrozenBlocks:
    def __init__(self, blocks, group=None, slots: int = 3):
        self.blocks = list(blocks)
        self.group = group
        self.world = get_world_size(group)
        self.rank = get_rank() if group is None else dist.get_rank(group)
        dev = next(self.blocks[0].parameters()).device
        self.device = dev
        self.cuda = dev.type == "cuda"
        self.layout = []  # per block: (params, offsets, numel, shard len, arena offset)
        off = 0
        for b in self.blocks:
            ps = [p for p in b.parameters() if not p.requires_grad and p.dtype == torch.bfloat16 and p.numel() > 0]
            offs, n = [], 0
            for p in ps:
                offs.append(n)
                n += -(-p.numel() // _ALIGN) * _ALIGN
            ln = max(64, -(-n // (self.world * 64)) * 64)
            self.layout.append((ps, offs, n, ln, off))
            off += ln
        self.arena = SymmBuffer(max(off, 64), torch.bfloat16, dev, group, zero=True)
        with torch.no_grad():
            for ps, offs, n, ln, base in self.layout:
                flat = torch.zeros(ln * self.world, dtype=torch.bfloat16, device=dev)
                for p, o in zip(ps, offs):
                    flat[o:o + p.numel()].copy_(p.data.reshape(-1))
                self.arena.tensor[base:base + ln].copy_(flat[self.rank * ln:(self.rank + 1) * ln])
                for p in ps:
                    p._fsdp_shape = tuple(p.shape)
                    p.data = torch.empty(0, dtype=p.dtype, device=dev)
        self.max_full = max(ln * self.world for _, _, _, ln, _ in self.layout)
        self.slots = [torch.empty(self.max_full, dtype=torch.bfloat16, device=dev) for _ in range(slots)]
        self.resident = [-1] * slots
        self.stream = torch.cuda.Stream(device=dev) if self.cuda else None
        self.done = [None] * slots
        self.last = None
        self.handles = [b.register_forward_pre_hook(self._make_pre(i)) for i, b in enumerate(self.blocks)]
        if self.cuda:
            torch.cuda.synchronize(dev)
        if is_distributed() and self.world > 1:
            barrier()  # every shard is in place before any peer reads it

    # ------------------------------------------------------------------ gather
    def _gather(self, i: int, slot: int):
        ps, offs, n, ln, base = self.layout[i]
        dst = self.slots[slot]
        if self.cuda:
            from ..ops import ext
            from ..runtime.nvtx import nvtx_range
            with nvtx_range(f"dmad.fsdp.gather[{i}]"):
                ext().fsdp_gather([p + base * 2 for p in self.arena.ptrs], dst, ln, n)
        elif is_distributed() and self.world > 1:
            parts = [torch.empty(ln, dtype=torch.bfloat16) for _ in range(self.world)]
            dist.all_gather(parts, self.arena.tensor[base:base + ln].contiguous(), group=self.group)
            dst[: ln * self.world].copy_(torch.cat(parts))
        else:
            dst[:ln].copy_(self.arena.tensor[base:base + ln])
        self.resident[slot] = i

    def _issue(self, i: int):
        """Gather block i into its slot on the side stream after the compute issued so far."""
        slot = i % len(self.slots)
        if not self.cuda:
            self._gather(i, slot)
            return
        ev = torch.cuda.Event()
        ev.record(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(self.stream):
            self.stream.wait_event(ev)
            self._gather(i, slot)
            done = torch.cuda.Event()
            done.record(self.stream)
        self.done[slot] = done

    def _bind(self, i: int, slot: int):
        ps, offs, _, _, _ = self.layout[i]
        buf = self.slots[slot]
        for p, o in zip(ps, offs):
            p.data = buf[o:o + _numel(p._fsdp_shape)].view(p._fsdp_shape)

    def _make_pre(self, i: int):
        def pre(module, args):
            slot = i % len(self.slots)
            if self.resident[slot] != i:
                self._issue(i)
            if self.cuda and self.done[slot] is not None:
                torch.cuda.current_stream(self.device).wait_event(self.done[slot])
            self._bind(i, slot)
            step = 1 if (self.last is None or i > self.last) else -1
            self.last = i
            nxt = i + step
            if 0 <= nxt < len(self.blocks) and self.resident[nxt % len(self.slots)] != nxt:
                self._issue(nxt)
        return pre

    def check_checkpointing(self, checkpointed: int):
        if checkpointed < len(self.blocks):
            raise ValueError("blocks with sharded weights must be activation-checkpointed when trained "
                             f"({checkpointed} of {len(self.blocks)} are)")

    def remove(self):
        for h in self.handles:
            h.remove()


def _numel(shape):
    n = 1
    for d in shape:
        n *= d
    return n
