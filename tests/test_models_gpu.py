"""Model-level checks on the GPU: the Wan DiT on the sm_100a kernels against the same
model run through the fp32 PyTorch math on CPU, and one DMAD generator + critic iteration."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_wan_forward_backward_matches_cpu():
    from dmad_b200.models.wan import WanConfig, WanModel
    torch.manual_seed(0)
    cfg = WanConfig(dim=256, ffn_dim=512, num_heads=2, num_layers=2, text_dim=128)
    m = WanModel(cfg)
    for p in m.parameters():
        p.data.normal_(0, 0.05)
    x = torch.randn(1, 16, 3, 12, 16)
    t = torch.tensor([[700.0]])
    c = torch.randn(1, 40, 128)
    ref = m(x, t, c)
    ref.square().mean().backward()
    g_ref = {n: p.grad.clone() for n, p in m.named_parameters()}
    m.zero_grad()
    mg = m.to("cuda", torch.bfloat16)
    out = mg(x.cuda(), t.cuda(), c.cuda().bfloat16())
    rel = ((out.float().cpu() - ref).norm() / ref.norm()).item()
    assert rel < 5e-2, rel
    out.float().square().mean().backward()
    for n, p in mg.named_parameters():
        gr = g_ref[n]
        if gr.norm() < 1e-6:
            continue
        r = ((p.grad.float().cpu() - gr).norm() / gr.norm()).item()
        assert r < 0.1, (n, r)


def test_wan_dmad_iterations():
    from dmad_b200 import ops
    from dmad_b200.distill.wan_dmad import WanDMAD, WanDMADConfig
    from dmad_b200.models.wan import WanConfig
    cfg = WanDMADConfig(net=WanConfig(dim=256, ffn_dim=512, num_heads=2, num_layers=2))
    m = WanDMAD(cfg, device="cuda", dtype=torch.bfloat16)
    shp = (1, 16, 3, 16, 16)
    batch = {"latents": torch.randn(shp, device="cuda"), "real_latents": torch.randn(shp, device="cuda"),
             "context": torch.randn(1, 512, 4096, device="cuda", dtype=torch.bfloat16)}
    for it in range(4):
        out = m.training_step(batch, it)
        for k, v in out.items():
            assert torch.isfinite(torch.as_tensor(float(v))), k
    torch.cuda.synchronize()
    ops.check_device_status()
    x = m.generate(batch["context"], shp)
    assert torch.isfinite(x).all()


def test_wan_forward_jvp_gpu_matches_cpu():
    from dmad_b200.models.wan import WanConfig, WanModel
    from dmad_b200.models.wan_jvp import wan_forward_jvp
    torch.manual_seed(0)
    cfg = WanConfig(dim=256, ffn_dim=512, num_heads=2, num_layers=2, text_dim=128)
    m = WanModel(cfg)
    for p in m.parameters():
        p.data.normal_(0, 0.05)
    x, tx = torch.randn(1, 16, 3, 8, 12), torch.randn(1, 16, 3, 8, 12)
    t, tt = torch.tensor([[600.0]]), torch.tensor([[25.0]])
    c = torch.randn(1, 40, 128)
    ref, tref = wan_forward_jvp(m, x, tx, t, tt, c)
    mg = m.to("cuda", torch.bfloat16)
    out, tout = wan_forward_jvp(mg, x.cuda(), tx.cuda(), t.cuda(), tt.cuda(), c.cuda().bfloat16())
    assert ((out.cpu() - ref).norm() / ref.norm()).item() < 5e-2
    assert ((tout.cpu() - tref).norm() / tref.norm()).item() < 5e-2


@pytest.mark.parametrize("lora", [0, 8])
def test_mm_only_checkpoint_keeps_kernel_outputs(lora):
    """mm_only on the CUDA path: the tcgen05 attention and LoRA-linear forwards are dispatcher ops whose
    outputs the recomputation reuses; gradients equal the unchecked run's."""
    from torch.utils._python_dispatch import TorchDispatchMode

    import dmad_b200.ops.linear  # noqa: F401  (registers dmad::lora_linear_fwd)
    from dmad_b200.models.wan import WanConfig, WanModel

    class Count(TorchDispatchMode):
        n = 0

        def __torch_dispatch__(self, func, types, args=(), kwargs=None):
            if func in (torch.ops.dmad.flash_attn_fwd.default, torch.ops.dmad.lora_linear_fwd.default):
                Count.n += 1
            return func(*args, **(kwargs or {}))

    def run(policy):
        torch.manual_seed(0)
        m = WanModel(WanConfig(dim=256, ffn_dim=512, num_heads=2, num_layers=2, text_dim=64, freq_dim=64))
        torch.nn.init.normal_(m.head.head.weight, std=0.05)
        if lora:
            m.enable_lora(lora)
            for b in m.blocks:
                for lin in b.linears():
                    torch.nn.init.normal_(lin.lora_B, std=0.02)
        m = m.cuda().to(torch.bfloat16).train()
        if policy:
            m.checkpoint_blocks, m.checkpoint_policy = 2, policy
        g = torch.Generator().manual_seed(4)
        x = torch.randn(1, 16, 2, 16, 16, generator=g).cuda()
        t, ctx = torch.rand(1, 1, generator=g).cuda(), torch.randn(1, 8, 64, generator=g).cuda()
        out = m(x, t, ctx)
        Count.n = 0
        with Count():
            out.float().square().mean().backward()
        return torch.cat([p.grad.float().reshape(-1) for p in m.parameters() if p.grad is not None]), Count.n

    g0, n0 = run(None)
    g1, n1 = run("mm_only")
    g2, n2 = run("block_wise")
    assert n0 == 0 and n1 == 0 and n2 > 0, (n0, n1, n2)
    for g in (g1, g2):
        assert ((g - g0).norm() / g0.norm()).item() < 1e-2
