"""Data-parallel gradient synchronisation over flat buckets.

Baseline path (NCCL): gradients are packed into ~256 MB buckets and all-reduced
(averaged) after backward; packing uses one copy kernel per bucket.  This is the
NCCL-only reference point for the fused reduce-scatter + AdamW kernel.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from .dist import get_world_size, is_distributed


class GradSync:
    def __init__(self, params, bucket_bytes: int = 256 << 20, group=None, enabled: bool = True):
        self.enabled = enabled
        self.params = [p for p in params if p.requires_grad]
        self.bucket_bytes = bucket_bytes
        self.group = group

    @torch.no_grad()
    def sync(self):
        if not self.enabled or not is_distributed() or get_world_size(self.group) == 1:
            return
        world = get_world_size(self.group)
        by_dtype: dict = {}
        for p in self.params:
            if p.grad is None:
                p.grad = torch.zeros_like(p)
            by_dtype.setdefault(p.grad.dtype, []).append(p)
        for _, ps in by_dtype.items():
            bucket, size = [], 0
            for p in ps + [None]:
                if p is not None:
                    bucket.append(p)
                    size += p.grad.numel() * p.grad.element_size()
                if bucket and (p is None or size >= self.bucket_bytes):
                    flat = torch.cat([q.grad.reshape(-1) for q in bucket])
                    dist.all_reduce(flat, op=dist.ReduceOp.SUM, group=self.group)
                    flat.div_(world)
                    off = 0
                    for q in bucket:
                        n = q.grad.numel()
                        q.grad.copy_(flat[off:off + n].view_as(q.grad))
                        off += n
                    bucket, size = [], 0
