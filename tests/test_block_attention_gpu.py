"""Block-masked attention on the tcgen05 kernels (a flash launch per key range, merged by LSE in the
epilogue; flash backward per range) against fp32 masked dense attention, forward and gradients."""
import math

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("mode,local,sink,qbo", [("block_causal", 0, 0, 0), ("block_causal", 2, 1, 1),
                                                 ("teacher_forcing", 2, 1, 0)])
def test_block_attention_cuda(mode, local, sink, qbo):
    from dmad_b200 import ops
    from dmad_b200.ops.block_attention import AttnMaskSpec, BlockPattern, block_attention, dense_mask

    pat = BlockPattern(frame_tokens=96, first_chunk_frames=1, chunk_frames=2)
    if mode == "teacher_forcing":
        spec = AttnMaskSpec(mode, pat, local, sink, 0, clean_blocks=3)
        Q = KV = 2 * pat.blocks_to_tokens(3)
    else:
        spec = AttnMaskSpec(mode, pat, local, sink, qbo)
        KV = pat.blocks_to_tokens(qbo + 4)
        Q = KV - pat.blocks_to_tokens(qbo)
    torch.manual_seed(0)
    B, H = 1, 2
    q = torch.randn(B, Q, H, 128, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    k = torch.randn(B, KV, H, 128, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    v = torch.randn(B, KV, H, 128, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    g = torch.randn(B, Q, H, 128, device="cuda", dtype=torch.bfloat16)
    out = block_attention(q, k, v, spec)
    out.backward(g)
    torch.cuda.synchronize()
    ops.check_device_status()
    qr, kr, vr = (t.detach().float().requires_grad_(True) for t in (q, k, v))
    m = dense_mask(spec, Q, KV, device="cuda")
    s = torch.einsum("bqhd,bkhd->bhqk", qr, kr) / math.sqrt(128)
    p = torch.nan_to_num(torch.softmax(s.masked_fill(~m, float("-inf")), -1))
    ref = torch.einsum("bhqk,bkhd->bqhd", p, vr)
    ref.backward(g.float())
    assert (out.float() - ref).abs().max().item() < 3e-2
    for a, b, name in ((q.grad, qr.grad, "dq"), (k.grad, kr.grad, "dk"), (v.grad, vr.grad, "dv")):
        rel = ((a.float() - b).norm() / b.norm()).item()
        assert rel < 2e-2, (name, rel)
