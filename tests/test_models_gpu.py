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
