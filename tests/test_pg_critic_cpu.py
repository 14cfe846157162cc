"""Pretrained-feature (Projected-GAN style) critic of the EDM stack: shapes and frozen parts of the
two-head critic, the EfficientNet-Lite0 feature network, and one EDM DMAD step with it
(parity: train/image/main/edm/pg_critic.py, edm_guidance.py:87-91,147-148,228-267)."""
import torch


def test_lite0_shapes_and_parameter_count():
    from dmad_b200.models.pg_critic import EfficientNetLite0

    net = EfficientNetLite0().eval()
    n = sum(p.numel() for p in net.parameters())
    assert 4.5e6 < n < 4.8e6, n  # EfficientNet-Lite0 has 4.65M parameters
    with torch.no_grad():
        assert net(torch.zeros(1, 3, 224, 224)).shape == (1, 1000)
        h = net.bn1(net.conv_stem(torch.zeros(1, 3, 224, 224)))
        for i, (c, r) in enumerate([(16, 112), (24, 56), (40, 28), (80, 14), (112, 14), (192, 7), (320, 7)]):
            h = net.blocks[i](h)
            assert h.shape[1:] == (c, r, r), (i, h.shape)


def test_two_head_critic_shapes_and_frozen_features():
    from dmad_b200.models.pg_critic import PGTwoHeadCritic

    torch.manual_seed(0)
    crit = PGTwoHeadCritic(("vgg16_bn", "tf_efficientnet_lite0"), c_dim=10).train()
    assert all(not p.requires_grad for p in crit.features.parameters())
    assert not crit.features.training and crit.heads_real.training
    x = torch.rand(2, 3, 32, 32) * 2 - 1
    c = torch.eye(10)[torch.tensor([1, 7])]
    d_r, d_t = crit(x, c)
    assert d_r.shape == d_t.shape and d_r.shape[0] == 2 and d_r.shape[1] > 4
    (d_r.mean() + d_t.mean()).backward()
    assert all(p.grad is None for p in crit.features.parameters())
    assert any(p.grad is not None for p in crit.heads_teacher.parameters())
    # the class embeddings start from the Lite0 classifier weight
    lite = crit.features["tf_efficientnet_lite0"].pretrained.net.classifier.weight
    assert torch.equal(crit.heads_real["vgg16_bn"].heads[0].embed.weight.detach(), lite.detach())


def test_edm_step_with_pretrained_critic():
    from dmad_b200.distill.edm_dmad import EDMDMAD, EDMDMADConfig
    from dmad_b200.models.edm import EDMPrecond

    torch.manual_seed(0)
    teacher = EDMPrecond(16, 3, label_dim=10, model_channels=16, channel_mult=(1, 2), num_blocks=1,
                         attn_resolutions=(8,))
    cfg = EDMDMADConfig(resolution=16, label_dim=10, batch_size=2, pretrained_critic="tf_efficientnet_lite0",
                        r1_gamma=0.1)
    m = EDMDMAD(cfg, teacher=teacher)
    out = m.train_step(m.synthetic_batch(torch.Generator().manual_seed(0)))
    for k in ("generator_loss", "critic_loss", "critic_acc_t", "r1"):
        assert torch.isfinite(torch.tensor(out[k])), k
    assert all(not p.requires_grad for p in m.critic.pg.features.parameters())
    # gap routing with per-pixel logits: per-sample means per band
    idx = torch.arange(0, 1000, 100)
    m.critic.update_gap(torch.linspace(0, 1, 10), torch.zeros(10), idx, idx)
    assert m.critic.gap_weight(idx) is not None
