"""Activation checkpointing policies for transformer blocks.

Parity: train/wan/rcm/utils/selective_activation_checkpoint.py:26-74.

* ``"block_wise"``: the whole block is recomputed in the backward; only its inputs are kept.
* ``"mm_only"``: the outputs of the matrix products are kept from the forward and everything else
  (normalisation, modulation, RoPE, activations, gates) is recomputed.  The kept ops are the
  library GEMMs (``aten.mm`` / ``addmm`` / ``bmm``), this package's tcgen05 flash-attention forward
  (``dmad::flash_attn_fwd``, output and LSE) and LoRA-fused linear (``dmad::lora_linear_fwd``).  The
  fused context-parallel attention (exchange + attention in one autograd function) is recomputed whole,
  as the reference recomputes its all-to-all.
"""
from __future__ import annotations

import functools

import torch
from torch.utils.checkpoint import CheckpointPolicy, checkpoint, create_selective_checkpoint_contexts

POLICIES = ("block_wise", "mm_only")


@functools.lru_cache(maxsize=1)
def _saved_ops():
    from ..ops import attention as _attn  # noqa: F401  (registers dmad::flash_attn_fwd)
    from ..ops import linear as _lin  # noqa: F401  (registers dmad::lora_linear_fwd)

    aten = torch.ops.aten
    return frozenset({aten.mm.default, aten.addmm.default, aten.bmm.default, aten.baddbmm.default,
                      torch.ops.dmad.flash_attn_fwd.default, torch.ops.dmad.lora_linear_fwd.default})


def _mm_only_policy(ctx, op, *args, **kwargs):
    return CheckpointPolicy.MUST_SAVE if op in _saved_ops() else CheckpointPolicy.PREFER_RECOMPUTE


def mm_only_context():
    return create_selective_checkpoint_contexts(_mm_only_policy)


def checkpoint_block(fn, *args, policy: str = "block_wise"):
    """``fn(*args)`` under activation checkpointing with the given policy (non-reentrant)."""
    if policy == "mm_only":
        return checkpoint(fn, *args, use_reentrant=False, context_fn=mm_only_context)
    if policy != "block_wise":
        raise ValueError(f"unknown checkpoint policy {policy!r} (one of {POLICIES})")
    return checkpoint(fn, *args, use_reentrant=False)
