"""Image DMAD paths on CPU: EDM config-1 step and a tiny SDXL-shaped step."""
import torch


def test_edm_config1_step():
    from dmad_b200.distill.edm_dmad import EDMDMAD, EDMDMADConfig
    torch.manual_seed(0)
    m = EDMDMAD(EDMDMADConfig(critic_sigma="lognormal", warmup_steps=0))
    b = m.synthetic_batch(torch.Generator().manual_seed(0))
    before = [p.detach().clone() for p in m.generator.parameters()]
    out = m.train_step(b)
    for k in ("generator_loss", "critic_loss", "critic_acc_t"):
        assert torch.isfinite(torch.tensor(out[k]))
    assert any(not torch.equal(a, p) for a, p in zip(before, m.generator.parameters()))
    # the critic is encoder-only with a one-logit head per sample
    d_r, d_t = m.critic.logits(b["real_image"], torch.ones(4), b["labels"])
    assert d_r.shape == (4,) and d_t.shape == (4,)


def test_edm_gap_routing_engages():
    from dmad_b200.distill.edm_dmad import EDMCritic, EDMDMADConfig
    from dmad_b200.models.edm import config1_unet
    c = EDMCritic(EDMDMADConfig(critic_spectral_norm=False), config1_unet())
    idx = torch.arange(0, 1000, 100)
    c.update_gap(torch.linspace(0, 1, 10), torch.zeros(10), idx, idx)
    w = c.gap_weight(idx)
    assert w is not None and w.shape == (10,) and float(w[0]) > float(w[-1])


def test_sdxl_tiny_step_and_full_size():
    from dmad_b200.distill.sdxl_dmad import SDXLDMAD, SDXLDMADConfig
    from dmad_b200.models.sdxl import SDXLUNet
    n = sum(p.numel() for p in SDXLUNet().parameters())
    assert 2.4e9 < n < 2.7e9
    cfg = SDXLDMADConfig(latent=32, sn_iters=3, unet_kwargs=dict(channels=(32, 64, 64), depths=(0, 1, 1), ctx_dim=32,
                                                                pooled_dim=16, addition_time_embed_dim=8))
    d = SDXLDMAD(cfg, device="cpu", dtype=torch.float32)
    B = 2
    b = {"noise": torch.randn(B, 4, 32, 32), "real": torch.randn(B, 4, 32, 32), "teacher": torch.randn(B, 4, 32, 32),
         "ctx": torch.randn(B, 7, 32), "pooled": torch.randn(B, 16)}
    out = d.train_step(b)
    assert all(torch.isfinite(v) for v in out.values())


def test_fold_spectral_norm_matches_normalised_forward():
    import copy
    from dmad_b200.distill.edm_dmad import sn_wrap
    from dmad_b200.tools.export_unet import fold_spectral_norm, plain_state_dict

    torch.manual_seed(0)
    net = torch.nn.Sequential(torch.nn.Conv2d(3, 8, 3, padding=1), torch.nn.SiLU(), torch.nn.Conv2d(8, 3, 3, padding=1))
    plain = copy.deepcopy(net)
    for m in net:
        if isinstance(m, torch.nn.Conv2d):
            sn_wrap(m, power_iters=20)
    net.eval()
    x = torch.randn(2, 3, 8, 8)
    ref = net(x)
    sd = plain_state_dict(net, torch.float32)
    assert not any("parametrizations" in k or k.endswith(("sn_u", "sn_v", "sn_gain")) for k in sd)
    plain.load_state_dict(sd)
    torch.testing.assert_close(plain(x), ref, rtol=1e-4, atol=1e-5)


def test_frozen_gain_spectral_norm_properties():
    """At set-up the normalised layer computes what the plain one did; after the weight changes its
    spectral norm is pulled back to the set-up value; the module deep-copies and round-trips its state."""
    import copy
    from dmad_b200.algorithms.spectral import SNLinear, apply_spectral_norm

    torch.manual_seed(0)
    net = torch.nn.Sequential(torch.nn.Linear(12, 9), torch.nn.SiLU(), torch.nn.Conv2d(3, 4, 3))
    plain = copy.deepcopy(net)
    assert apply_spectral_norm(net, power_iters=50) == 2
    assert isinstance(net[0], SNLinear)
    x = torch.randn(5, 12)
    torch.testing.assert_close(net[0](x), plain[0](x), rtol=1e-4, atol=1e-5)
    s0 = torch.linalg.matrix_norm(plain[0].weight, ord=2)
    with torch.no_grad():
        net[0].weight.mul_(3.0).add_(0.1 * torch.randn_like(net[0].weight))
    for _ in range(60):  # power steps in training mode converge to the new sigma
        w_eff = net[0].sn_weight()
    torch.testing.assert_close(torch.linalg.matrix_norm(w_eff.detach(), ord=2), s0, rtol=1e-3, atol=1e-4)
    twin = copy.deepcopy(net)
    twin.load_state_dict(net.state_dict())
    net.eval(), twin.eval()
    torch.testing.assert_close(twin[0](x), net[0](x))
    # gradients reach the raw weight through sigma
    net.train()
    net[0](x).sum().backward()
    assert net[0].weight.grad is not None and torch.isfinite(net[0].weight.grad).all()


def test_sdxl_generator_ema_weight_decay_and_clip():
    """The SDXL trainer's optimiser settings of the reference (AdamW weight decay, clipping at
    max_grad_norm) and its generator EMA: the exported EMA follows the half-life recursion of the weights
    after every step, on both data-parallel optimiser paths."""
    import copy
    import os
    import tempfile

    from dmad_b200.distill.sdxl_dmad import SDXLDMAD, SDXLDMADConfig
    for dp in ("sharded", "nccl"):
        cfg = SDXLDMADConfig(latent=32, sn_iters=3, dp_optimizer=dp, generator_lr=1e-3, ema_kimg=0.001,
                             max_grad_norm=1.0,
                             unet_kwargs=dict(channels=(32, 64, 64), depths=(0, 1, 1), ctx_dim=32, pooled_dim=16,
                                              addition_time_embed_dim=8))
        d = SDXLDMAD(cfg, device="cpu", dtype=torch.float32)
        ema = [p.detach().clone() for p in d.gen_params]
        B = 2
        g = torch.Generator().manual_seed(1)
        for _ in range(3):
            b = {"noise": torch.randn(B, 4, 32, 32, generator=g), "real": torch.randn(B, 4, 32, 32, generator=g),
                 "teacher": torch.randn(B, 4, 32, 32, generator=g), "ctx": torch.randn(B, 7, 32, generator=g),
                 "pooled": torch.randn(B, 16, generator=g)}
            decay = d.ema_decay(B)
            d.train_step(b)
            ema = [e * decay + p.detach() * (1 - decay) for e, p in zip(ema, d.gen_params)]
        for a, b_ in zip(d.ema_params(), ema):
            torch.testing.assert_close(a.reshape(b_.shape).float(), b_, rtol=1e-4, atol=1e-6)
        assert any(not torch.equal(a.reshape(p.shape), p.detach()) for a, p in zip(d.ema_params(), d.gen_params))
        with tempfile.TemporaryDirectory() as tmp:
            d.export_emas(tmp)
            sd = torch.load(os.path.join(tmp, "pytorch_model_ema.bin"))
        assert sd.keys() == d.generator.state_dict().keys()
        net = copy.deepcopy(d.generator)
        net.load_state_dict(sd)


def test_sdxl_one_step_mode_and_warmup():
    """The one-step variant (pure noise in at the conditioning timestep) trains, and the learning rate
    ramps from 0 over the warm-up steps (the first update leaves the generator unchanged)."""
    from dmad_b200.distill.sdxl_dmad import SDXLDMAD, SDXLDMADConfig
    cfg = SDXLDMADConfig(latent=32, sn_iters=3, conditioning_timestep=399, warmup_steps=2, generator_lr=1e-3,
                         unet_kwargs=dict(channels=(32, 64, 64), depths=(0, 1, 1), ctx_dim=32, pooled_dim=16,
                                          addition_time_embed_dim=8))
    d = SDXLDMAD(cfg, device="cpu", dtype=torch.float32)
    before = [p.detach().clone() for p in d.gen_params]
    B = 2
    b = {"noise": torch.randn(B, 4, 32, 32), "real": torch.randn(B, 4, 32, 32), "teacher": torch.randn(B, 4, 32, 32),
         "ctx": torch.randn(B, 7, 32), "pooled": torch.randn(B, 16)}
    out = d.train_step(b)
    assert all(torch.isfinite(v) for v in out.values())
    assert all(torch.equal(a, p.detach()) for a, p in zip(before, d.gen_params))
    d.train_step(b)
    assert abs(d.opt_g.lr - 0.5 * cfg.generator_lr) < 1e-12
    assert any(not torch.equal(a, p.detach()) for a, p in zip(before, d.gen_params))
