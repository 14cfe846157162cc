"""Flash-attention JVP forward (csrc/flash_jvp.cu) against fp32 PyTorch: O, tO, LSE, zero-tangent
variants, a rescale-heavy case, and the gradient of O through the plain flash backward.
The oracle is the forward-mode derivative of naive fp32 attention (torch.func.jvp), as the
reference's inline test of its Triton kernel does."""
import math

import pytest
import torch

pytestmark = pytest.mark.gpu

dev = "cuda"


def _rand(*shape, s=1.0):
    return (torch.randn(*shape, device=dev) * s).to(torch.bfloat16)


def _oracle(q, k, v, tq, tk, tv, scale):
    def f(q_, k_, v_):
        s = torch.einsum("blhd,bmhd->bhlm", q_, k_) * scale
        return torch.einsum("bhlm,bmhd->blhd", torch.softmax(s, -1), v_)

    z = lambda t, ref: t.float() if t is not None else torch.zeros_like(ref.float())  # noqa: E731
    o, to = torch.func.jvp(f, (q.float(), k.float(), v.float()), (tq.float(), z(tk, k), z(tv, v)))
    s = torch.einsum("blhd,bmhd->bhlm", q.float(), k.float()) * scale
    return o, to, torch.logsumexp(s, -1)


@pytest.mark.parametrize("B,Lq,Lk,H,has_tk,has_tv", [
    (1, 128, 128, 1, True, True), (1, 256, 384, 2, True, True), (2, 999, 999, 2, True, True),
    (1, 1000, 512, 3, False, False), (1, 300, 77, 2, True, False), (1, 2048, 2048, 1, False, True)])
def test_flash_jvp_matches_fp32(B, Lq, Lk, H, has_tk, has_tv):
    from dmad_b200 import ops

    torch.manual_seed(0)
    q, k, v = _rand(B, Lq, H, 128), _rand(B, Lk, H, 128), _rand(B, Lk, H, 128)
    tq = _rand(B, Lq, H, 128, s=0.5)
    tk = _rand(B, Lk, H, 128, s=0.5) if has_tk else None
    tv = _rand(B, Lk, H, 128, s=0.5) if has_tv else None
    scale = 1 / math.sqrt(128)
    e = ops.ext()
    o = torch.empty_like(q)
    to = torch.empty_like(q)
    lse = torch.empty(B, H, e.flash_lse_pad(Lq), device=dev)
    e.flash_jvp_fwd(q, k, v, tq, tk, tv, o, to, lse, scale)
    torch.cuda.synchronize()
    ops.check_device_status()
    ro, rto, rlse = _oracle(q, k, v, tq, tk, tv, scale)
    assert (o.float() - ro).abs().max().item() < 2e-2
    t_err = (to.float() - rto).abs().max().item()
    assert t_err < 3e-2 * max(1.0, rto.abs().max().item()), t_err
    lse_nat = lse[:, :, :Lq] / math.log2(math.e)
    assert (lse_nat - rlse).abs().max().item() < 2e-3
    assert torch.isinf(lse[:, :, Lq:]).all()


def test_flash_jvp_rescale_path():
    """Logits whose row maxima grow along the keys exercise the lazy O~ / T~ rescale."""
    from dmad_b200 import ops

    torch.manual_seed(1)
    B, L, H = 1, 1024, 2
    q = _rand(B, L, H, 128, s=2.0)
    ramp = torch.linspace(0.2, 3.0, L, device=dev).view(1, L, 1, 1)
    k = (torch.randn(B, L, H, 128, device=dev) * ramp).to(torch.bfloat16)
    v, tq, tk, tv = _rand(B, L, H, 128), _rand(B, L, H, 128, s=0.3), _rand(B, L, H, 128, s=0.3), _rand(B, L, H, 128)
    o, to = ops.flash_attention_jvp(q, k, v, tq, tk, tv)
    torch.cuda.synchronize()
    ops.check_device_status()
    ro, rto, _ = _oracle(q, k, v, tq, tk, tv, 1 / math.sqrt(128))
    assert (o.float() - ro).abs().max().item() < 3e-2
    rel = (to.float() - rto).norm() / rto.norm()
    assert rel.item() < 1e-2, rel.item()


def test_flash_jvp_grad_of_o_matches_flash_attention():
    from dmad_b200 import ops

    torch.manual_seed(2)
    B, L, H = 1, 640, 2
    q, k, v = (_rand(B, L, H, 128).requires_grad_(True) for _ in range(3))
    tq, tk, tv = (_rand(B, L, H, 128, s=0.5) for _ in range(3))
    do = _rand(B, L, H, 128)
    o, to = ops.flash_attention_jvp(q, k, v, tq, tk, tv)
    assert not to.requires_grad
    g1 = torch.autograd.grad(o, (q, k, v), do)
    o2 = ops.flash_attention(q, k, v)
    g2 = torch.autograd.grad(o2, (q, k, v), do)
    torch.testing.assert_close(o, o2, rtol=0, atol=1e-2)
    for a, b in zip(g1, g2):
        torch.testing.assert_close(a.float(), b.float(), rtol=2e-2, atol=2e-2)


@pytest.mark.parametrize("Lq,blocks,has_tk", [(999, (256, 300, 443), True), (512, (128, 77), False)])
def test_flash_jvp_accumulate_over_key_blocks(Lq, blocks, has_tk):
    """The blockwise (ring) form: key blocks visited one launch at a time and merged in the
    epilogue reproduce the JVP over all keys."""
    from dmad_b200 import ops

    torch.manual_seed(1)
    B, H, Lk = 1, 2, sum(blocks)
    q, k, v = _rand(B, Lq, H, 128), _rand(B, Lk, H, 128), _rand(B, Lk, H, 128)
    tq, tv = _rand(B, Lq, H, 128, s=0.5), _rand(B, Lk, H, 128, s=0.5)
    tk = _rand(B, Lk, H, 128, s=0.5) if has_tk else None
    scale = 1 / math.sqrt(128)
    e = ops.ext()
    o, to = torch.empty_like(q), torch.empty_like(q)
    lse = torch.empty(B, H, e.flash_lse_pad(Lq), device=dev)
    acc_o = torch.empty(B, Lq, H, 128, device=dev)
    acc_u = torch.empty_like(acc_o)
    acc_lse, acc_mu = torch.empty_like(lse), torch.empty_like(lse)
    s0 = 0
    for i, n in enumerate(blocks):
        sl = slice(s0, s0 + n)
        s0 += n
        e.flash_jvp_accumulate(q, k[:, sl].contiguous(), v[:, sl].contiguous(), tq,
                               tk[:, sl].contiguous() if tk is not None else None, tv[:, sl].contiguous(), o, to, lse,
                               acc_o, acc_u, acc_lse, acc_mu, i > 0, i == len(blocks) - 1, scale)
    torch.cuda.synchronize()
    ops.check_device_status()
    ro, rto, rlse = _oracle(q, k, v, tq, tk, tv, scale)
    assert (o.float() - ro).abs().max().item() < 2e-2
    t_err = (to.float() - rto).abs().max().item()
    assert t_err < 3e-2 * max(1.0, rto.abs().max().item()), t_err
    assert (lse[:, :, :Lq] / math.log2(math.e) - rlse).abs().max().item() < 2e-3
    assert torch.isinf(lse[:, :, Lq:]).all()
