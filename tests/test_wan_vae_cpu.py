"""Wan-shaped causal VAE on CPU: shapes (1 + 4k frames <-> 1 + k latents, stride 8), causality
(changing frame t never changes outputs before t), parameter count of the 2.1 configuration, and
the reference's checkpoint key layout."""
import torch


def _small():
    from dmad_b200.models.wan_vae import WanVAEModel

    torch.manual_seed(0)
    return WanVAEModel(dim=8, z_dim=4, dim_mult=(1, 2, 2, 2), num_res_blocks=1)


def test_shapes_and_roundtrip_shapes():
    from dmad_b200.models.wan_vae import WanVAE

    m = _small()
    vae = WanVAE(model=m)
    vae.mean, vae.std = torch.zeros(1, 4, 1, 1, 1), torch.ones(1, 4, 1, 1, 1)
    x = torch.rand(1, 3, 9, 32, 48) * 2 - 1
    z = vae.encode(x)
    assert z.shape == (1, 4, 3, 4, 6)
    y = vae.decode(z)
    assert y.shape == (1, 3, 9, 32, 48)
    assert WanVAE.latent_frames(81) == 21 and WanVAE.pixel_frames(21) == 81


def test_causal_in_time():
    m = _small()
    x = torch.randn(1, 3, 9, 16, 16)
    x2 = x.clone()
    x2[:, :, 5:] += 1.0  # change frames 5.. (latent frames 2.. start at pixel frame 5)
    with torch.no_grad():
        z1, z2 = m.encoder(x), m.encoder(x2)
        assert torch.equal(z1[:, :, :2], z2[:, :, :2]) and not torch.equal(z1[:, :, 2:], z2[:, :, 2:])
        zz = torch.randn(1, 4, 3, 2, 2)
        zz2 = zz.clone()
        zz2[:, :, 2] += 1.0
        d1, d2 = m.decoder(zz), m.decoder(zz2)
        assert torch.equal(d1[:, :, :5], d2[:, :, :5]) and not torch.equal(d1[:, :, 5:], d2[:, :, 5:])


def test_wan21_config_size_and_keys():
    from dmad_b200.models.wan_vae import WanVAEModel

    with torch.device("meta"):
        m = WanVAEModel()
    n = sum(p.numel() for p in m.parameters())
    assert 120e6 < n < 135e6, n
    keys = set(m.state_dict())
    for k in ("encoder.conv1.weight", "encoder.downsamples.0.residual.0.gamma",
              "encoder.downsamples.0.residual.2.weight", "encoder.middle.1.to_qkv.weight", "encoder.head.2.weight",
              "conv1.weight", "conv2.weight", "decoder.upsamples.3.resample.1.weight",
              "decoder.upsamples.3.time_conv.weight", "decoder.head.0.gamma"):
        assert k in keys, k
