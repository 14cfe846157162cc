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


@pytest.mark.parametrize("mode", ["block_causal", "teacher_forcing"])
def test_block_attention_jvp_cuda(mode):
    """Masked JVP on the tcgen05 JVP kernel (accumulated over key ranges) against fp32 torch.func.jvp of
    masked dense attention."""
    from dmad_b200 import ops
    from dmad_b200.ops.block_attention import AttnMaskSpec, BlockPattern, block_attention_jvp, dense_mask

    pat = BlockPattern(frame_tokens=96, first_chunk_frames=1, chunk_frames=2)
    if mode == "teacher_forcing":
        spec = AttnMaskSpec(mode, pat, 2, 1, 0, clean_blocks=3)
        Q = KV = 2 * pat.blocks_to_tokens(3)
    else:
        spec = AttnMaskSpec(mode, pat, 2, 1)
        Q = KV = pat.blocks_to_tokens(4)
    torch.manual_seed(1)
    mk = lambda n, s=1.0: (torch.randn(1, n, 2, 128, device="cuda") * s).to(torch.bfloat16)  # noqa: E731
    q, k, v, tq, tk, tv = mk(Q), mk(KV), mk(KV), mk(Q, 0.5), mk(KV, 0.5), mk(KV, 0.5)
    o, to = block_attention_jvp(q, k, v, tq, tk, tv, spec)
    torch.cuda.synchronize()
    ops.check_device_status()
    m = dense_mask(spec, Q, KV, device="cuda")

    def f(q_, k_, v_):
        s = torch.einsum("bqhd,bkhd->bhqk", q_, k_) / math.sqrt(128)
        p = torch.nan_to_num(torch.softmax(s.masked_fill(~m, float("-inf")), -1))
        return torch.einsum("bhqk,bkhd->bqhd", p, v_)

    ro, rto = torch.func.jvp(f, (q.float(), k.float(), v.float()), (tq.float(), tk.float(), tv.float()))
    assert (o.float() - ro).abs().max().item() < 3e-2
    assert ((to.float() - rto).norm() / rto.norm()).item() < 2e-2
