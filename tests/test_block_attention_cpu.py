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


@pytest.mark.parametrize("mode", ["block_causal", "teacher_forcing"])
def test_block_attention_jvp_matches_autodiff(mode):
    """The masked JVP (per query block over its key ranges) equals torch.func.jvp of the masked
    dense attention."""
    from dmad_b200.ops.block_attention import block_attention_jvp

    torch.manual_seed(1)
    pat = BlockPattern(frame_tokens=4, first_chunk_frames=1, chunk_frames=2)
    if mode == "teacher_forcing":
        spec = AttnMaskSpec(mode, pat, local_attn_blocks=2, sink_blocks=1, clean_blocks=3)
        Q = KV = 2 * pat.blocks_to_tokens(3)
    else:
        spec = AttnMaskSpec(mode, pat, local_attn_blocks=2, sink_blocks=1)
        Q = KV = pat.blocks_to_tokens(4)
    q, tq = torch.randn(1, Q, 2, 16, dtype=torch.float64), torch.randn(1, Q, 2, 16, dtype=torch.float64)
    k, tk = torch.randn(1, KV, 2, 16, dtype=torch.float64), torch.randn(1, KV, 2, 16, dtype=torch.float64)
    v, tv = torch.randn(1, KV, 2, 16, dtype=torch.float64), torch.randn(1, KV, 2, 16, dtype=torch.float64)
    m = dense_mask(spec, Q, KV)

    def f(q_, k_, v_):
        s = torch.einsum("bqhd,bkhd->bhqk", q_, k_) / math.sqrt(16)
        p = torch.nan_to_num(torch.softmax(s.masked_fill(~m, float("-inf")), -1))
        return torch.einsum("bhqk,bkhd->bqhd", p, v_)

    ro, rto = torch.func.jvp(f, (q, k, v), (tq, tk, tv))
    o, to = block_attention_jvp(q, k, v, tq, tk, tv, spec)
    torch.testing.assert_close(o, ro)
    torch.testing.assert_close(to, rto)


def test_wan_forward_jvp_with_block_mask_matches_autodiff():
    from dmad_b200.models.wan import WanConfig, WanModel
    from dmad_b200.models.wan_jvp import wan_forward_jvp

    torch.manual_seed(0)
    m = WanModel(WanConfig(dim=128, ffn_dim=256, num_heads=2, num_layers=2, text_dim=32, freq_dim=64)).double()
    torch.nn.init.normal_(m.head.head.weight, std=0.05)
    g = torch.Generator().manual_seed(2)
    x, tx = torch.randn(1, 16, 3, 4, 8, generator=g).double(), torch.randn(1, 16, 3, 4, 8, generator=g).double()
    t, tt = torch.rand(1, 1, generator=g).double(), torch.rand(1, 1, generator=g).double()
    ctx = torch.randn(1, 6, 32, generator=g).double()
    spec = AttnMaskSpec("block_causal", BlockPattern(frame_tokens=8, first_chunk_frames=1, chunk_frames=1))
    out, tout = wan_forward_jvp(m, x, tx, t, tt, ctx, attn_meta=spec)
    with torch.no_grad():
        ref = m(x, t, ctx, attn_meta=spec)
        eps = 1e-3  # central differences of the (fp32) network output
        fd = (m(x + eps * tx, t + eps * tt, ctx, attn_meta=spec).double() -
              m(x - eps * tx, t - eps * tt, ctx, attn_meta=spec).double()) / (2 * eps)
    torch.testing.assert_close(out.double(), ref.double(), rtol=1e-5, atol=1e-6)  # parts of the JVP path run in fp32
    rel = ((tout.double() - fd).norm() / fd.norm()).item()
    assert rel < 1e-3, rel
