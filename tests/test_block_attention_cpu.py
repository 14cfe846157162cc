"""Block masks as key ranges (ops/block_attention.py): the rectangles of ``mask_ranges`` reproduce the
reference's element predicate for block-causal (windows, sinks, query offsets) and teacher-forcing
masks, and the range-merged attention equals masked dense softmax attention with its gradients."""
import itertools
import math

import pytest
import torch

from dmad_b200.ops.block_attention import AttnMaskSpec, BlockPattern, block_attention, dense_mask, mask_ranges


def _from_ranges(spec, Q, KV):
    m = torch.zeros(Q, KV, dtype=torch.bool)
    for q0, q1, rng in mask_ranges(spec, Q, KV):
        for a, b in rng:
            assert not m[q0:q1, a:b].any(), "ranges of one query block overlap"
            m[q0:q1, a:b] = True
    return m


def _specs():
    for ft, fc, cf in itertools.product((3, 5), (1, 2), (1, 3)):
        pat = BlockPattern(frame_tokens=ft, first_chunk_frames=fc, chunk_frames=cf)
        for local, sink in itertools.product((0, 1, 2, 3), (0, 1, 2)):
            for qbo in (0, 1, 2):
                prefix = pat.blocks_to_tokens(qbo)
                Q = pat.blocks_to_tokens(qbo + 4) - prefix - 1  # a ragged last block
                yield AttnMaskSpec("block_causal", pat, local, sink, qbo), Q, prefix + Q
            for clean in (2, 3):
                n = pat.blocks_to_tokens(clean)
                yield AttnMaskSpec("teacher_forcing", pat, local, sink, 0, clean), 2 * n, 2 * n


def test_ranges_match_reference_predicate():
    n = 0
    for spec, Q, KV in _specs():
        torch.testing.assert_close(_from_ranges(spec, Q, KV), dense_mask(spec, Q, KV), msg=str(spec))
        n += 1
    assert n > 100


@pytest.mark.parametrize("mode", ["block_causal", "teacher_forcing", "none"])
def test_block_attention_matches_masked_dense(mode):
    torch.manual_seed(0)
    pat = BlockPattern(frame_tokens=4, first_chunk_frames=1, chunk_frames=2)
    if mode == "teacher_forcing":
        spec = AttnMaskSpec(mode, pat, local_attn_blocks=2, sink_blocks=1, clean_blocks=3)
        Q = KV = 2 * pat.blocks_to_tokens(3)
    else:
        spec = AttnMaskSpec(mode, pat, local_attn_blocks=2, sink_blocks=1, q_block_offset=1)
        KV = pat.blocks_to_tokens(4)
        Q = KV - pat.blocks_to_tokens(1)
    q = torch.randn(2, Q, 2, 16, dtype=torch.float64, requires_grad=True)
    k = torch.randn(2, KV, 2, 16, dtype=torch.float64, requires_grad=True)
    v = torch.randn(2, KV, 2, 16, dtype=torch.float64, requires_grad=True)
    out = block_attention(q, k, v, spec)
    m = dense_mask(spec, Q, KV)
    s = torch.einsum("bqhd,bkhd->bhqk", q, k) / math.sqrt(16)
    s = s.masked_fill(~m, float("-inf"))
    p = torch.nan_to_num(torch.softmax(s, -1))
    ref = torch.einsum("bhqk,bkhd->bqhd", p, v)
    torch.testing.assert_close(out, ref)
    g = torch.randn_like(ref)
    gb = torch.autograd.grad(out, (q, k, v), g)
    gr = torch.autograd.grad(ref, (q, k, v), g)
    for a, b in zip(gb, gr):
        torch.testing.assert_close(a, b)
