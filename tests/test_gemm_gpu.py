"""tcgen05 GEMM (csrc/gemm.cu) and the LoRA-fused linear against fp32 PyTorch: tails in M / N / K,
bias, GELU epilogue, the extra K panel, and the autograd of the LoRA linear."""
import pytest
import torch

pytestmark = pytest.mark.gpu
dev = "cuda"


def _r(*s, scale=1.0):
    return (torch.randn(*s, device=dev) * scale).to(torch.bfloat16)


@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (1000, 1536, 1536), (77, 392, 200), (4099, 520, 1032)])
@pytest.mark.parametrize("act", [0, 1])
def test_gemm_matches_fp32(M, N, K, act):
    from dmad_b200 import ops

    torch.manual_seed(0)
    a, b = _r(M, K), _r(N, K, scale=K ** -0.5)
    bias = torch.randn(N, device=dev)
    d = torch.empty(M, N, device=dev, dtype=torch.bfloat16)
    ops.ext().gemm_bf16(a, b, None, None, bias, d, 1.0, act)
    torch.cuda.synchronize()
    ops.check_device_status()
    ref = a.float() @ b.float().t() + bias
    if act == 1:
        ref = torch.nn.functional.gelu(ref, approximate="tanh")
    assert (d.float() - ref).abs().max().item() < 3e-2 * max(1.0, ref.abs().max().item())


def test_gemm_extra_k_panel_and_strided_output():
    from dmad_b200 import ops

    torch.manual_seed(1)
    M, N, K, r = 600, 768, 512, 128
    a, b, a2, b2 = _r(M, K), _r(N, K, scale=0.05), _r(M, r), _r(N, r, scale=0.05)
    big = torch.zeros(M, N + 64, device=dev, dtype=torch.bfloat16)
    d = big[:, 32:32 + N]
    ops.ext().gemm_bf16(a, b, a2, b2, None, d, 0.5, 0)
    torch.cuda.synchronize()
    ref = 0.5 * (a.float() @ b.float().t() + a2.float() @ b2.float().t())
    assert (d.float() - ref).abs().max().item() < 2e-2 * max(1.0, ref.abs().max().item())
    assert big[:, :32].abs().max().item() == 0 and big[:, 32 + N:].abs().max().item() == 0


def test_lora_linear_forward_backward():
    from dmad_b200.ops.linear import lora_linear

    torch.manual_seed(2)
    M, N, K, r, s = 300, 512, 384, 128, 0.5
    x = _r(2, M // 2, K).requires_grad_(True)
    w = _r(N, K, scale=0.05)
    bias = _r(N)
    a = _r(r, K, scale=0.05).requires_grad_(True)
    b = _r(N, r, scale=0.05).requires_grad_(True)
    y = lora_linear(x, w, bias, a, b, s)
    g = _r(*y.shape)
    dx, da, db = torch.autograd.grad(y, (x, a, b), g)
    xf, af, bf = (t.detach().float().requires_grad_(True) for t in (x, a, b))
    yr = xf @ w.float().t() + bias.float() + s * (xf @ af.t()) @ bf.t()
    rdx, rda, rdb = torch.autograd.grad(yr, (xf, af, bf), g.float())
    assert (y.float() - yr).abs().max().item() < 3e-2
    for got, ref in ((dx, rdx), (da, rda), (db, rdb)):
        assert ((got.float() - ref).norm() / ref.norm()).item() < 1e-2


def test_seglinear_lora_uses_fused_path():
    from dmad_b200.models.layers import SegLinear

    torch.manual_seed(3)
    lin = SegLinear(256, [("q", 256), ("k", 256), ("v", 256)], flat_name="qkv").to(dev, torch.bfloat16)
    lin.enable_lora(128)
    with torch.no_grad():
        lin.lora_B.normal_(0, 0.02)
    x = _r(64, 256)
    y = lin(x)
    w = lin.weight.float()
    ref = x.float() @ w.t() + lin.bias.float() + lin.lora_scale * (x.float() @ lin.lora_A.float().t()) @ \
        (lin.lora_B * lin.lora_mask).float().t()
    assert (y.float() - ref).abs().max().item() < 3e-2


@pytest.mark.parametrize("a_mn,b_mn", [(False, True), (True, False), (True, True)])
@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (304, 520, 1000), (384, 1536, 4104)])
def test_gemm_transposed_operands(a_mn, b_mn, M, N, K):
    """Operands read MN-major (stored transposed) give A B^T as the K-major ones do."""
    from dmad_b200 import ops

    torch.manual_seed(3)
    a, b = _r(M, K), _r(N, K, scale=K ** -0.5)
    d = torch.empty(M, N, device=dev, dtype=torch.bfloat16)
    ops.ext().gemm_bf16_ex(a.t().contiguous() if a_mn else a, b.t().contiguous() if b_mn else b, None, None, None,
                           d, None, 1.0, 0, a_mn, b_mn, 1)
    torch.cuda.synchronize()
    ops.check_device_status()
    ref = a.float() @ b.float().t()
    assert (d.float() - ref).abs().max().item() < 3e-2 * max(1.0, ref.abs().max().item())


@pytest.mark.parametrize("split", [1, 3, 16, 40])
def test_gemm_split_k_fp32(split):
    """Split-K with fp32 reduction in the epilogue: p^T q over a long token dimension (the LoRA weight
    gradients), including splits that get no K steps."""
    from dmad_b200 import ops

    torch.manual_seed(4)
    T, m, n = 4100, 128, 1536
    p, q = _r(T, m, scale=0.1), _r(T, n, scale=0.1)
    out = torch.zeros(m, n, device=dev)
    ops.ext().gemm_bf16_ex(p, q, None, None, None, None, out, 2.0, 0, True, True, split)
    torch.cuda.synchronize()
    ops.check_device_status()
    ref = 2.0 * p.float().t() @ q.float()
    assert (out - ref).abs().max().item() < 1e-2 * max(1.0, ref.abs().max().item())


def test_lora_linear_backward_on_tcgen05_matches_fp32_at_wan_shape():
    """The LoRA-linear backward (dX with the extra K panel, dA / dB split-K) at a Wan FFN shape."""
    from dmad_b200.ops.linear import lora_linear

    torch.manual_seed(5)
    M, N, K, r, s = 4096, 8960, 1536, 128, 1.0
    x = _r(M, K).requires_grad_(True)
    w = _r(N, K, scale=K ** -0.5)
    a = _r(r, K, scale=K ** -0.5).requires_grad_(True)
    b = _r(N, r, scale=0.02).requires_grad_(True)
    y = lora_linear(x, w, None, a, b, s)
    g = _r(*y.shape, scale=0.1)
    dx, da, db = torch.autograd.grad(y, (x, a, b), g)
    torch.cuda.synchronize()
    from dmad_b200 import ops
    ops.check_device_status()
    xf, af, bf = (t.detach().float().requires_grad_(True) for t in (x, a, b))
    yf = xf @ w.float().t() + s * (xf @ af.t()) @ bf.t()
    rdx, rda, rdb = torch.autograd.grad(yf, (xf, af, bf), g.float())
    for got, ref in ((dx, rdx), (da, rda), (db, rdb)):
        rel = ((got.float() - ref).norm() / ref.norm()).item()
        assert rel < 2e-2, rel
