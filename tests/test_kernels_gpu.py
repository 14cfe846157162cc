"""sm_100a kernels against fp32 PyTorch references (small and odd shapes)."""
import math

import pytest
import torch

pytestmark = pytest.mark.gpu

dev = "cuda"


def _ext():
    from dmad_b200 import ops
    assert ops.native_available(), "extension must be built for GPU tests"
    return ops.ext()


def _attn_ref(q, k, v, scale):
    qf, kf, vf = (t.float().transpose(1, 2) for t in (q, k, v))
    s = qf @ kf.transpose(-1, -2) * scale
    return (torch.softmax(s, -1) @ vf).transpose(1, 2), torch.logsumexp(s, -1)


@pytest.mark.parametrize("B,Lq,Lk,H", [(1, 128, 128, 1), (1, 256, 256, 2), (2, 999, 999, 2), (1, 1000, 512, 3),
                                       (1, 4095, 4095, 1), (1, 77, 300, 2)])
def test_flash_fwd(B, Lq, Lk, H):
    e = _ext()
    torch.manual_seed(0)
    q = torch.randn(B, Lq, H, 128, device=dev, dtype=torch.bfloat16)
    k = torch.randn(B, Lk, H, 128, device=dev, dtype=torch.bfloat16)
    v = torch.randn(B, Lk, H, 128, device=dev, dtype=torch.bfloat16)
    scale = 1 / math.sqrt(128)
    o = torch.empty_like(q)
    lse = torch.empty(B, H, e.flash_lse_pad(Lq), device=dev)
    e.flash_fwd(q, k, v, o, lse, scale)
    torch.cuda.synchronize()
    from dmad_b200 import ops
    ops.check_device_status()
    ref, ref_lse = _attn_ref(q, k, v, scale)
    err = (o.float() - ref).abs().max().item()
    assert err < 2e-2, err
    lse_nat = lse[:, :, :Lq] * math.log(2)
    assert (lse_nat - ref_lse).abs().max().item() < 1e-2


def test_flash_fwd_strided_qkv():
    """q/k/v as views of one fused [B, L, 3, H, 128] projection (the model's layout)."""
    e = _ext()
    B, L, H = 1, 700, 2
    qkv = torch.randn(B, L, 3 * H * 128, device=dev, dtype=torch.bfloat16)
    q = qkv[..., :H * 128].view(B, L, H, 128)
    k = qkv[..., H * 128:2 * H * 128].view(B, L, H, 128)
    v = qkv[..., 2 * H * 128:].view(B, L, H, 128)
    o = torch.empty(B, L, H, 128, device=dev, dtype=torch.bfloat16)
    lse = torch.empty(B, H, e.flash_lse_pad(L), device=dev)
    e.flash_fwd(q, k, v, o, lse, 0.1)
    ref, _ = _attn_ref(q, k, v, 0.1)
    assert (o.float() - ref).abs().max().item() < 2e-2


@pytest.mark.parametrize("B,Lq,Lk,H", [(1, 128, 128, 1), (1, 384, 256, 2), (1, 999, 999, 1), (2, 300, 512, 2)])
def test_flash_bwd(B, Lq, Lk, H):
    from dmad_b200.ops import flash_attention
    torch.manual_seed(1)
    q = torch.randn(B, Lq, H, 128, device=dev, dtype=torch.bfloat16, requires_grad=True)
    k = torch.randn(B, Lk, H, 128, device=dev, dtype=torch.bfloat16, requires_grad=True)
    v = torch.randn(B, Lk, H, 128, device=dev, dtype=torch.bfloat16, requires_grad=True)
    g = torch.randn(B, Lq, H, 128, device=dev, dtype=torch.bfloat16)
    o = flash_attention(q, k, v)
    o.backward(g)
    qr, kr, vr = (t.detach().float().requires_grad_(True) for t in (q, k, v))
    ref, _ = _attn_ref(qr, kr, vr, 1 / math.sqrt(128))
    ref.backward(g.float())
    from dmad_b200 import ops
    ops.check_device_status()
    for a, b, name in ((q.grad, qr.grad, "dq"), (k.grad, kr.grad, "dk"), (v.grad, vr.grad, "dv")):
        rel = (a.float() - b).norm() / b.norm()
        assert rel < 2e-2, (name, rel.item())


@pytest.mark.parametrize("B,Lq,Lk,H", [(1, 128, 128, 1), (2, 999, 999, 3), (1, 4096, 4096, 2), (2, 1024, 77, 4),
                                       (1, 300, 700, 2)])
def test_flash_head_dim_64(B, Lq, Lk, H):
    """Head dim 64 (the SDXL U-Net's): forward O and LSE, and dQ / dK / dV, against fp32 autograd;
    Lk = 77 is the text cross-attention."""
    from dmad_b200 import ops
    e = ops.ext()
    torch.manual_seed(4)
    q = torch.randn(B, Lq, H, 64, device=dev, dtype=torch.bfloat16, requires_grad=True)
    k = torch.randn(B, Lk, H, 64, device=dev, dtype=torch.bfloat16, requires_grad=True)
    v = torch.randn(B, Lk, H, 64, device=dev, dtype=torch.bfloat16, requires_grad=True)
    g = torch.randn(B, Lq, H, 64, device=dev, dtype=torch.bfloat16)
    scale = 1 / math.sqrt(64)
    o_, lse = torch.empty_like(q), torch.empty(B, H, e.flash_lse_pad(Lq), device=dev)
    e.flash_fwd(q.detach(), k.detach(), v.detach(), o_, lse, scale)
    o = ops.flash_attention(q, k, v)
    o.backward(g)
    torch.cuda.synchronize()
    ops.check_device_status()
    qr, kr, vr = (t.detach().float().requires_grad_(True) for t in (q, k, v))
    ref, ref_lse = _attn_ref(qr, kr, vr, scale)
    ref.backward(g.float())
    assert (o.float() - ref).abs().max().item() < 2e-2
    assert torch.equal(o, o_)
    assert ((lse[:, :, :Lq] * math.log(2)) - ref_lse).abs().max().item() < 1e-2
    for a, b, name in ((q.grad, qr.grad, "dq"), (k.grad, kr.grad, "dk"), (v.grad, vr.grad, "dv")):
        rel = (a.float() - b).norm() / b.norm()
        assert rel < 2e-2, (name, rel.item())


def test_sdxl_attention_module_on_flash_kernels():
    """The SDXL Attention block (10 heads of 64) on CUDA against its CPU SDPA path, self and cross."""
    from dmad_b200.models.sdxl import Attention
    torch.manual_seed(5)
    for ctx_dim in (None, 2048):
        m = Attention(640, ctx_dim)
        x = torch.randn(2, 1024, 640)
        ctx = torch.randn(2, 77, 2048) if ctx_dim else None
        ref = m(x, ctx)
        mc = m.to(dev, torch.bfloat16)
        out = mc(x.to(dev, torch.bfloat16), ctx.to(dev, torch.bfloat16) if ctx is not None else None)
        rel = (out.float().cpu() - ref).norm() / ref.norm()
        assert rel < 2e-2, (ctx_dim, rel.item())


@pytest.mark.parametrize("B,Lq,Lk,H", [(1, 128, 128, 1), (1, 384, 256, 2), (1, 999, 999, 1), (2, 300, 512, 2),
                                        (1, 1000, 1300, 3)])
def test_flash_bwd_fused(B, Lq, Lk, H):
    """The single-kernel backward (fp32 dQ accumulator) against fp32 autograd, writing into strided
    slices of one [B, L, 3, H, 128] buffer as the fused-QKV layers do."""
    from dmad_b200 import ops
    e = ops.ext()
    torch.manual_seed(2)
    q = torch.randn(B, Lq, H, 128, device=dev, dtype=torch.bfloat16)
    k = torch.randn(B, Lk, H, 128, device=dev, dtype=torch.bfloat16)
    v = torch.randn(B, Lk, H, 128, device=dev, dtype=torch.bfloat16)
    g = torch.randn(B, Lq, H, 128, device=dev, dtype=torch.bfloat16)
    scale = 1 / math.sqrt(128)
    o = torch.empty_like(q)
    lse = torch.empty(B, H, e.flash_lse_pad(Lq), device=dev)
    e.flash_fwd(q, k, v, o, lse, scale)
    dq = torch.empty(B, Lq, 3, H, 128, device=dev, dtype=torch.bfloat16)[:, :, 1]
    dk, dv = torch.empty_like(k), torch.empty_like(v)
    acc = torch.full((B * H * lse.shape[-1] * 128,), float("nan"), device=dev)
    e.flash_bwd_fused(q, k, v, o, g, lse, dq, dk, dv, torch.empty_like(lse), acc, scale)
    torch.cuda.synchronize()
    ops.check_device_status()
    qr, kr, vr = (t.detach().float().requires_grad_(True) for t in (q, k, v))
    ref, _ = _attn_ref(qr, kr, vr, scale)
    ref.backward(g.float())
    for a, b, name in ((dq, qr.grad, "dq"), (dk, kr.grad, "dk"), (dv, vr.grad, "dv")):
        rel = (a.float() - b).norm() / b.norm()
        assert rel < 2e-2, (name, rel.item())


@pytest.mark.parametrize("D,R,G", [(1536, 1000, 2), (5120, 257, 1), (256, 64, 4)])
@pytest.mark.parametrize("rms", [False, True])
def test_ln_mod(D, R, G, rms):
    from dmad_b200.ops.norm import ln_mod, ln_mod_reference
    torch.manual_seed(2)
    x = torch.randn(R, D, device=dev, dtype=torch.bfloat16, requires_grad=True)
    a = (0.1 * torch.randn(G, D, device=dev)).requires_grad_(True)
    c = (0.1 * torch.randn(G, D, device=dev)).requires_grad_(True)
    rpg = (R + G - 1) // G
    y = ln_mod(x, a, c, 1.0, rpg, None, 1e-6, rms)
    xr, ar, cr = (t.detach().clone().float().requires_grad_(True) for t in (x, a, c))
    yr = ln_mod_reference(xr, ar, cr, 1.0, rpg, None, 1e-6, rms).float()
    assert (y.float() - yr).abs().max().item() < 3e-2
    gy = torch.randn_like(y)
    y.backward(gy)
    yr.backward(gy.float())
    assert ((x.grad.float() - xr.grad).norm() / xr.grad.norm()).item() < 1e-2
    assert ((a.grad - ar.grad).norm() / ar.grad.norm()).item() < 1e-2
    assert ((c.grad - cr.grad).norm() / cr.grad.norm()).item() < 1e-2


@pytest.mark.parametrize("D,R,G", [(1536, 999, 3), (5120, 130, 2), (128, 77, 5)])
@pytest.mark.parametrize("rms", [False, True])
def test_ln_mod_bwd_fusions_and_row_groups(D, R, G, rms):
    """The backward kernels with an explicit per-row group index (groups interleaved, so the column sums
    change group many times inside a row tile), the residual-gradient addend and the gated-residual
    fusion, against fp32 PyTorch."""
    from dmad_b200 import ops
    e = ops.ext()
    torch.manual_seed(7)
    x = torch.randn(R, D, device=dev, dtype=torch.bfloat16)
    dy = torch.randn(R, D, device=dev, dtype=torch.bfloat16)
    dres = torch.randn(R, D, device=dev, dtype=torch.bfloat16)
    yg = torch.randn(R, D, device=dev, dtype=torch.bfloat16)
    a = 0.1 * torch.randn(G, D, device=dev)
    gate = torch.randn(G, D, device=dev)
    gidx = (torch.arange(R, device=dev) * 7 // 5 % G).int()
    xf = x.float()
    mean = None if rms else xf.mean(1)
    var = (xf * xf).mean(1) if rms else xf.var(1, unbiased=False)
    rstd = torch.rsqrt(var + 1e-6)
    dx = torch.empty_like(x)
    dyg = torch.empty_like(x)
    da = torch.zeros(G, D, device=dev)
    dc = torch.zeros(G, D, device=dev)
    dgate = torch.zeros(G, D, device=dev)
    e.ln_mod_bwd(dy, x, mean, rstd, a, 1.0, R, gidx, rms, dx, dres, da, dc, gate, yg, dyg, dgate)
    torch.cuda.synchronize()
    ops.check_device_status()
    g = gidx.long()
    n = (xf - (0.0 if rms else mean[:, None])) * rstd[:, None]
    A = 1.0 + a[g]
    dn = dy.float() * A
    mdn = 0.0 if rms else dn.mean(1, keepdim=True)
    ref_dx = rstd[:, None] * (dn - mdn - n * (dn * n).mean(1, keepdim=True)) + dres.float()
    ref_da = torch.zeros(G, D, device=dev).index_add_(0, g, dy.float() * n)
    ref_dc = torch.zeros(G, D, device=dev).index_add_(0, g, dy.float())
    ref_dyg = ref_dx * gate[g]
    ref_dgate = torch.zeros(G, D, device=dev).index_add_(0, g, ref_dx * yg.float())
    for got, ref, name in ((dx, ref_dx, "dx"), (dyg, ref_dyg, "dyg"), (da, ref_da, "da"), (dc, ref_dc, "dc"),
                           (dgate, ref_dgate, "dgate")):
        rel = (got.float() - ref).norm() / ref.norm()
        assert rel < 1e-2, (name, rel.item())


def test_gate_residual():
    from dmad_b200.ops import gate_residual
    R, D, G = 600, 1536, 3
    x = torch.randn(R, D, device=dev, dtype=torch.bfloat16, requires_grad=True)
    y = torch.randn(R, D, device=dev, dtype=torch.bfloat16, requires_grad=True)
    gt = torch.randn(G, D, device=dev, requires_grad=True)
    out = gate_residual(x, y, gt, rows_per_group=R // G)
    g = torch.arange(R, device=dev) // (R // G)
    ref = x.float() + y.float() * gt[g]
    # one bf16 rounding of the output: relative error <= 2^-8
    assert ((out.float() - ref).abs() / ref.abs().clamp_min(1.0)).max().item() < 8e-3
    go = torch.randn_like(out)
    out.backward(go)
    assert torch.allclose(x.grad.float(), go.float())
    dy_ref = go.float() * gt[g].detach()
    assert ((y.grad.float() - dy_ref).abs() / dy_ref.abs().clamp_min(1.0)).max().item() < 8e-3
    ref_dg = torch.zeros(G, D, device=dev).index_add_(0, g, go.float() * y.detach().float())
    assert ((gt.grad - ref_dg).norm() / ref_dg.norm()).item() < 1e-3


def test_qk_norm_rope_and_attention_core():
    from dmad_b200.models.layers import self_attention_core
    from dmad_b200.models.wan import rope_3d_angles
    torch.manual_seed(3)
    B, T, Hh, Ww, H = 1, 3, 6, 10, 2
    L, D = T * Hh * Ww, 2 * 128
    ang = rope_3d_angles(T, Hh, Ww, 128, device=dev)
    cos, sin = torch.cos(ang), torch.sin(ang)
    qkv = torch.randn(B * L, 3 * D, device=dev, dtype=torch.bfloat16, requires_grad=True)
    wq = (1 + 0.1 * torch.randn(D, device=dev)).requires_grad_(True)
    wk = (1 + 0.1 * torch.randn(D, device=dev)).requires_grad_(True)
    out = self_attention_core(qkv, wq, wk, cos, sin, B, L, H)
    ref = self_attention_core(qkv.detach().cpu().float().requires_grad_(True), wq.detach().cpu().requires_grad_(True),
                              wk.detach().cpu().requires_grad_(True), cos.cpu(), sin.cpu(), B, L, H)
    assert (out.float().cpu() - ref.float()).abs().max().item() < 3e-2
    g = torch.randn_like(out)
    out.backward(g)
    qkv_r = qkv.detach().cpu().float().requires_grad_(True)
    wq_r, wk_r = wq.detach().cpu().requires_grad_(True), wk.detach().cpu().requires_grad_(True)
    ref = self_attention_core(qkv_r, wq_r, wk_r, cos.cpu(), sin.cpu(), B, L, H)
    ref.float().backward(g.float().cpu())
    assert ((qkv.grad.float().cpu() - qkv_r.grad).norm() / qkv_r.grad.norm()).item() < 3e-2
    assert ((wq.grad.cpu() - wq_r.grad).norm() / wq_r.grad.norm()).item() < 3e-2


def test_rope_roundtrip():
    from dmad_b200.ops.norm import rope_apply, rope_reference
    x = torch.randn(500, 256, device=dev, dtype=torch.bfloat16)
    ang = torch.rand(500, 64, device=dev) * 6
    y = rope_apply(x, torch.cos(ang), torch.sin(ang), 128)
    yr = rope_reference(x, torch.cos(ang), torch.sin(ang), 128)
    assert (y.float() - yr.float()).abs().max().item() < 3e-2
    z = rope_apply(y, torch.cos(ang), torch.sin(ang), 128, inverse=True)
    assert (z.float() - x.float()).abs().max().item() < 5e-2


def test_gelu():
    from dmad_b200.ops import gelu_tanh
    x = torch.randn(1000, 64, device=dev, dtype=torch.bfloat16, requires_grad=True)
    y = gelu_tanh(x)
    xr = x.detach().float().requires_grad_(True)
    yr = torch.nn.functional.gelu(xr, approximate="tanh")
    assert (y.float() - yr).abs().max().item() < 2e-2
    y.backward(torch.ones_like(y))
    yr.backward(torch.ones_like(yr))
    assert (x.grad.float() - xr.grad).abs().max().item() < 2e-2


def test_adamw_matches_torch():
    from dmad_b200.ops.optim import FusedAdamW
    torch.manual_seed(4)
    ps = [torch.nn.Parameter(torch.randn(n, device=dev).to(torch.bfloat16)) for n in (1000, 70000)]
    ref = [torch.nn.Parameter(p.detach().float().clone()) for p in ps]
    ema = [p.detach().float().clone() for p in ps]
    opt = FusedAdamW(ps, lr=1e-3, betas=(0.9, 0.99), eps=1e-8, weight_decay=0.01, ema=ema)
    ropt = torch.optim.AdamW(ref, lr=1e-3, betas=(0.9, 0.99), eps=1e-8, weight_decay=0.01)
    ema_ref = [p.detach().clone() for p in ref]
    for step in range(3):
        gs = [torch.randn_like(r) for r in ref]
        for p, r, g in zip(ps, ref, gs):
            p.grad = g.to(torch.bfloat16)
            r.grad = g.to(torch.bfloat16).float()
        opt.step(ema_beta=0.9)
        ropt.step()
        for er, r in zip(ema_ref, ref):
            er.mul_(0.9).add_(r.detach(), alpha=0.1)
    for m, r in zip(opt.master, ref):
        assert (m - r).abs().max().item() < 1e-5
    for e_, er in zip(ema, ema_ref):
        assert (e_ - er).abs().max().item() < 1e-5


def test_temb_kernels():
    from dmad_b200.ops import sinusoidal_embedding, small_linear
    t = torch.tensor([0.0, 13.0, 999.0], device=dev)
    s = sinusoidal_embedding(t, 256)
    sr = sinusoidal_embedding(t.cpu(), 256)
    assert (s.cpu() - sr).abs().max().item() < 1e-5
    x = torch.randn(3, 1536, device=dev)
    w = torch.randn(4000, 1536, device=dev, dtype=torch.bfloat16) * 0.02
    b = torch.randn(4000, device=dev)
    y = small_linear(x, w, b, act_in="silu")
    yr = torch.nn.functional.linear(torch.nn.functional.silu(x), w.float(), b)
    assert (y - yr).abs().max().item() < 1e-3


def test_flash_fwd_accumulate_merges_key_blocks():
    """Attention over keys split into three blocks, merged by the accumulate epilogue, equals the
    attention over all keys (output and log2 LSE)."""
    e = _ext()
    torch.manual_seed(4)
    B, Lq, H = 1, 300, 2
    q = torch.randn(B, Lq, H, 128, device=dev, dtype=torch.bfloat16)
    ks = [torch.randn(B, n, H, 128, device=dev, dtype=torch.bfloat16) for n in (256, 100, 384)]
    vs = [torch.randn_like(k) for k in ks]
    scale = 1 / math.sqrt(128)
    o = torch.empty_like(q)
    lse = torch.empty(B, H, e.flash_lse_pad(Lq), device=dev)
    acc = torch.empty(B, Lq, H, 128, device=dev)
    acc_lse = torch.empty_like(lse)
    for j, (k, v) in enumerate(zip(ks, vs)):
        e.flash_fwd_accumulate(q, k, v, o, lse, acc, acc_lse, j > 0, j == 2, scale)
    torch.cuda.synchronize()
    from dmad_b200 import ops
    ops.check_device_status()
    ref, ref_lse = _attn_ref(q, torch.cat(ks, 1), torch.cat(vs, 1), scale)
    assert (o.float() - ref).abs().max().item() < 2e-2
    assert (lse[:, :, :Lq] / math.log2(math.e) - ref_lse).abs().max().item() < 2e-3


def test_peer_copy_local():
    e = _ext()
    src = torch.randn(1000, device=dev)
    dst = torch.empty_like(src)
    e.peer_copy(dst, src.data_ptr(), src.numel() * 4)
    dst2 = torch.empty_like(src)
    e.peer_copy_to(dst2.data_ptr(), src, src.numel() * 4)
    torch.cuda.synchronize()
    assert torch.equal(dst, src) and torch.equal(dst2, src)


def test_fsdp_gather_single_rank():
    e = _ext()
    shard = torch.randn(1024, device=dev).to(torch.bfloat16)
    dst = torch.empty(1024, device=dev, dtype=torch.bfloat16)
    e.fsdp_gather([shard.data_ptr()], dst, 1024, 1000)
    torch.cuda.synchronize()
    assert torch.equal(dst[:1000], shard[:1000])


@pytest.mark.parametrize("world,ln", [(2, 1 << 20), (3, 40000), (8, 65536 + 8)])
def test_fsdp_gather_many_shards(world, ln):
    """Several shard addresses (here all on this GPU) and a grid-stride range larger than the grid:
    every element of the gathered buffer comes from its own shard exactly once."""
    e = _ext()
    shards = [torch.randn(ln, device=dev).to(torch.bfloat16) for _ in range(world)]
    n = ln * world - 8
    dst = torch.full((ln * world,), float("nan"), device=dev, dtype=torch.bfloat16)
    e.fsdp_gather([s.data_ptr() for s in shards], dst, ln, n)
    torch.cuda.synchronize()
    assert torch.equal(dst[:n], torch.cat(shards)[:n])
