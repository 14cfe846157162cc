"""Forward-mode JVP of the Wan DiT and the rCM objectives on CPU."""
import pytest
import torch

from dmad_b200.models.wan import WanConfig, WanModel
from dmad_b200.models.wan_jvp import attention_jvp, wan_forward_jvp


def test_attention_jvp_matches_autograd_jvp():
    torch.manual_seed(0)
    q, k, v, tq, tk, tv = (torch.randn(1, 70, 2, 16, dtype=torch.float64) for _ in range(6))

    def f(q, k, v):
        s = torch.einsum("bqhd,bkhd->bhqk", q, k) / 4.0
        return torch.einsum("bhqk,bkhd->bqhd", torch.softmax(s, -1), v)

    ref, tref = torch.func.jvp(f, (q, k, v), (tq, tk, tv))
    o, to = attention_jvp(q, k, v, tq, tk, tv, scale=0.25)
    assert torch.allclose(o.double(), ref, atol=1e-5) and torch.allclose(to.double(), tref, atol=1e-4)


def test_wan_forward_jvp_matches_torch_func_jvp():
    torch.manual_seed(0)
    cfg = WanConfig(dim=128, ffn_dim=256, num_heads=1, num_layers=2, text_dim=32)
    m = WanModel(cfg)
    for p in m.parameters():
        p.data.normal_(0, 0.05)
    x = torch.randn(1, 16, 2, 4, 6)
    t = torch.tensor([[400.0]])
    c = torch.randn(1, 8, 32)
    tx, tt = torch.randn_like(x), torch.tensor([[20.0]])
    ref, tref = torch.func.jvp(lambda a, b: m(a, b, c), (x, t), (tx, tt))
    out, tout = wan_forward_jvp(m, x, tx, t, tt, c)
    assert ((out - ref).norm() / ref.norm()) < 1e-5
    assert ((tout - tref).norm() / tref.norm()) < 1e-5


@pytest.mark.parametrize("kw", [dict(loss_scale=100.0), dict(loss_scale=100.0, use_rf_scm=True),
                                dict(loss_scale=100.0, cm_type="dcm"), dict(critic_mode="dmd")])
def test_rcm_objectives_run(kw):
    from dmad_b200.distill.wan_dmad import WanDMAD, WanDMADConfig
    cfg = WanConfig(dim=64, ffn_dim=128, num_heads=1, num_layers=1, text_dim=16)
    m = WanDMAD(WanDMADConfig(net=cfg, **kw), device="cpu", dtype=torch.float32)
    b = {"latents": torch.randn(1, 16, 2, 4, 4), "real_latents": torch.randn(1, 16, 2, 4, 4),
         "context": torch.randn(1, 8, 16)}
    for it in range(3):
        out = m.training_step(b, it)
        assert all(torch.isfinite(torch.as_tensor(float(v))) for v in out.values())


@pytest.mark.parametrize("use_ema", [False, True])
def test_generate_records_no_autograd_graph(use_ema):
    """Few-step sampling runs without autograd, with and without the EMA weights swapped in."""
    from dmad_b200.distill.wan_dmad import WanDMAD, WanDMADConfig

    cfg = WanConfig(dim=128, ffn_dim=256, num_heads=1, num_layers=2, text_dim=32)
    m = WanDMAD(WanDMADConfig(net=cfg, sn_power_iters=2), device="cpu", dtype=torch.float32)
    x = m.generate(torch.randn(1, 8, 32), (1, 16, 2, 4, 6), num_steps=2, use_ema=use_ema)
    assert x.shape == (1, 16, 2, 4, 6)
    assert not x.requires_grad and x.grad_fn is None
