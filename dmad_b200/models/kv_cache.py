"""Key/value cache for causal (block-by-block) generation with the Wan network.

Parity: train/wan/rcm/utils/kv_cache.py:10-225 -- ``KVCacheMode`` (disabled / append / readonly),
``KVCache`` (a preallocated [B, max_len, H, D] buffer per layer, committed chunks, ``get`` by chunk
count, ``write_transient``, ``compact_``), ``AttnContext`` per layer and ``CausalInferenceState`` for a
forward pass.  Keys are stored after qk-norm and RoPE (the rotation of a cached key never changes), in
the layout the attention kernels read, so attending to the cache is one more key range for the flash
kernel and needs no concatenation: the current chunk's keys are written behind the committed prefix
and the kernel reads the prefix plus the chunk as one contiguous view.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from enum import Enum

import torch

from ..ops.block_attention import AttnMaskSpec, BlockPattern


class KVCacheMode(str, Enum):
    DISABLED = "disabled"  # plain forward
    APPEND = "append"      # commit this chunk's K/V, attend to cache + chunk
    READONLY = "readonly"  # attend to cache + chunk without committing it


class KVCache:
    def __init__(self, max_len: int):
        self.max_len = int(max_len)
        self.k = self.v = None
        self.cur = 0
        self._cum_ends: list[int] = []

    def reset(self, free_buffers: bool = True):
        if free_buffers:
            self.k = self.v = None
        self.cur = 0
        self._cum_ends = []

    def ensure(self, B: int, H: int, D: int, dtype, device):
        if self.k is None:
            self.k = torch.empty((B, self.max_len, H, D), dtype=dtype, device=device)
            self.v = torch.empty_like(self.k)

    def append(self, k: torch.Tensor, v: torch.Tensor) -> tuple[int, int]:
        B, s, H, D = k.shape
        if self.cur + s > self.max_len:
            raise RuntimeError(f"KV cache overflow: {self.cur} + {s} > {self.max_len}")
        self.ensure(B, H, D, k.dtype, k.device)
        start, end = self.cur, self.cur + s
        self.k[:, start:end].copy_(k.detach())
        self.v[:, start:end].copy_(v.detach())
        self.cur = end
        self._cum_ends.append(end)
        return start, end

    def get_prefix_end(self, block_range: int | None = None) -> int:
        """End of the committed prefix: all of it (None), none (0) or the first ``block_range`` chunks."""
        if block_range is None:
            return self.cur
        if block_range < 0:
            raise ValueError(f"block_range must be >= 0, got {block_range}")
        if block_range == 0:
            return 0
        if block_range > len(self._cum_ends):
            raise IndexError(f"block_range={block_range} exceeds the {len(self._cum_ends)} cached chunks")
        return self._cum_ends[block_range - 1]

    def get(self, block_range: int | None = None):
        end = self.get_prefix_end(block_range)
        if end == 0 or self.k is None:
            return None, None
        return self.k[:, :end], self.v[:, :end]

    def write_transient(self, k: torch.Tensor, v: torch.Tensor, at: int):
        """Write K/V at ``at`` without committing; returns the views [0, at + s)."""
        B, s, H, D = k.shape
        if at + s > self.max_len:
            raise RuntimeError(f"KV cache overflow: {at} + {s} > {self.max_len}")
        self.ensure(B, H, D, k.dtype, k.device)
        self.k[:, at:at + s].copy_(k.detach())
        self.v[:, at:at + s].copy_(v.detach())
        return self.k[:, :at + s], self.v[:, :at + s]

    def compact_(self, keep_indices: torch.Tensor | None):
        """Keep the cached tokens at ``keep_indices`` ([n] shared or [B, n] per sample)."""
        if self.k is None or self.cur == 0 or keep_indices is None:
            return
        idx = keep_indices.to(self.k.device, torch.long)
        if idx.numel() and (int(idx.min()) < 0 or int(idx.max()) >= self.cur):
            raise IndexError(f"KV compact indices out of bounds for {self.cur} cached tokens")
        if idx.ndim == 1:
            k_new, v_new = self.k.index_select(1, idx), self.v.index_select(1, idx)
        elif idx.ndim == 2:
            g = idx[:, :, None, None].expand(-1, -1, self.k.shape[2], self.k.shape[3])
            k_new, v_new = torch.gather(self.k[:, :self.cur], 1, g), torch.gather(self.v[:, :self.cur], 1, g)
        else:
            raise ValueError(f"keep_indices must be 1-D or 2-D, got {idx.ndim}-D")
        n = k_new.shape[1]
        self.k[:, :n].copy_(k_new)
        self.v[:, :n].copy_(v_new)
        self.cur = n
        self._cum_ends = [n] if n else []

    @property
    def current_len(self) -> int:
        return self.cur


@dataclass
class AttnContext:
    """What one self-attention layer does with the cache in this forward."""

    mode: KVCacheMode = KVCacheMode.DISABLED
    kv_cache: KVCache | None = None
    block_range: int | None = None  # committed chunks visible to this chunk (None = all)
    mask: AttnMaskSpec | None = None  # mask of the chunk against (visible prefix + chunk)


@dataclass
class CausalInferenceState:
    """Per-layer caches and the position of the current chunk for causal generation."""

    num_layers: int
    max_len: int
    pattern: BlockPattern
    local_attn_blocks: int = 0
    sink_blocks: int = 0
    caches: list = field(default_factory=list)
    mode: KVCacheMode = KVCacheMode.READONLY
    block_idx: int = 0  # absolute block index of the current chunk

    def __post_init__(self):
        if not self.caches:
            self.caches = [KVCache(self.max_len) for _ in range(self.num_layers)]

    def frame_offset(self) -> int:
        return self.pattern.blocks_to_frames(self.block_idx)

    def context(self, layer: int) -> AttnContext:
        spec = AttnMaskSpec("block_causal", self.pattern, self.local_attn_blocks, self.sink_blocks, self.block_idx)
        return AttnContext(self.mode, self.caches[layer], self.block_idx, spec)

    def reset(self):
        for c in self.caches:
            c.reset()
        self.block_idx = 0
