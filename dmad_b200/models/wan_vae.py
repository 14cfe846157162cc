"""Wan2.1-shaped causal video VAE (stride 4 x 8 x 8, 16 latent channels).

Architecture and checkpoint key layout of the reference tokenizer (train/wan/rcm/tokenizers/
wan2pt1.py:37-740): causal 3-D convolutions (zero history before frame 0), channel RMS norms
with a learned gain, residual blocks, per-frame single-head attention in the middle blocks,
spatial resamplers (``downsample2d`` / ``upsample2d``) and temporal ones (``downsample3d``: the
first frame passes through, later frames are reduced by a stride-2 temporal convolution;
``upsample3d``: the first latent frame maps to one frame, every later frame to two through a
causal temporal convolution with its own zero history).  Configuration of the 2.1 VAE: base
96 channels, multipliers [1, 2, 4, 4], two residual blocks per level, temporal downsampling on the
last two levels.  ``WanVAE.encode`` / ``decode`` apply the published per-channel latent
normalisation (``LATENT_MEAN`` / ``LATENT_STD``, the latent format of Wan2.1 checkpoints).

Execution differs from the reference, which streams chunks of 1, 4, 4, ... frames through feature
caches: here each causal layer sees the whole clip at once, which is the same computation as the
cached streaming (a cache holds exactly the past frames a causal layer reads).  Convolutions and attention are cuDNN / PyTorch SDPA: the
VAE is outside the timed DiT path.
"""
from __future__ import annotations

import torch
import torch.nn as nn
import torch.nn.functional as F

# Wan2.1 latent normalisation (per latent channel)
LATENT_MEAN = [-0.7571, -0.7089, -0.9113, 0.1075, -0.1745, 0.9653, -0.1517, 1.5508,
               0.4134, -0.0715, 0.5517, -0.3632, -0.1922, -0.9497, 0.2503, -0.2921]
LATENT_STD = [2.8184, 1.4541, 2.3275, 2.6558, 1.2196, 1.7708, 2.6052, 2.0743,
              3.2687, 2.1526, 2.8652, 1.5579, 1.6382, 1.1253, 2.8251, 1.9160]


class CausalConv3d(nn.Conv3d):
    """Conv3d with all temporal padding on the past side (frame t sees frames <= t).

    ``history``: optional [B, C, h, H, W] input frames preceding ``x`` (streaming); otherwise zeros."""

    def __init__(self, *args, **kwargs):
        super().__init__(*args, **kwargs)
        pt, ph, pw = self.padding
        self.t_pad = 2 * pt
        self.sp_pad = (pw, pw, ph, ph)
        self.padding = (0, 0, 0)

    def forward(self, x, history=None):
        pad_t = self.t_pad
        if pad_t > 0 and history is not None and history.shape[2] > 0:
            h = history[:, :, -pad_t:].to(x.dtype)
            x = torch.cat([h, x], dim=2)
            pad_t -= h.shape[2]
        return super().forward(F.pad(x, self.sp_pad + (pad_t, 0)))


class RMSNormC(nn.Module):
    """x / ||x||_channels * sqrt(C) * gamma (+ bias), over dim 1."""

    def __init__(self, dim, images=True, bias=False):
        super().__init__()
        shape = (dim, 1, 1) if images else (dim, 1, 1, 1)
        self.scale = dim ** 0.5
        self.gamma = nn.Parameter(torch.ones(shape))
        self.bias = nn.Parameter(torch.zeros(shape)) if bias else None

    def forward(self, x):
        y = F.normalize(x, dim=1) * self.scale * self.gamma
        return y + self.bias if self.bias is not None else y


def _frames2d(fn, x):
    """Apply a 2-D module to every frame of [B, C, T, H, W]."""
    B, C, T, H, W = x.shape
    y = fn(x.transpose(1, 2).reshape(B * T, C, H, W))
    return y.reshape(B, T, *y.shape[1:]).transpose(1, 2)


class Resample(nn.Module):
    def __init__(self, dim, mode):
        super().__init__()
        self.mode = mode
        if mode in ("upsample2d", "upsample3d"):
            self.resample = nn.Sequential(nn.Upsample(scale_factor=(2.0, 2.0), mode="nearest-exact"),
                                          nn.Conv2d(dim, dim // 2, 3, padding=1))
            if mode == "upsample3d":
                self.time_conv = CausalConv3d(dim, dim * 2, (3, 1, 1), padding=(1, 0, 0))
        elif mode in ("downsample2d", "downsample3d"):
            self.resample = nn.Sequential(nn.ZeroPad2d((0, 1, 0, 1)), nn.Conv2d(dim, dim, 3, stride=(2, 2)))
            if mode == "downsample3d":
                self.time_conv = CausalConv3d(dim, dim, (3, 1, 1), stride=(2, 1, 1), padding=(0, 0, 0))
        else:
            self.resample = nn.Identity()

    def forward(self, x):
        if self.mode == "upsample3d" and x.shape[2] > 1:
            # frame 0 passes through; frames 1.. are doubled by a causal conv with zero history
            B, C, T, H, W = x.shape
            rest = self.time_conv(x[:, :, 1:])                       # [B, 2C, T-1, H, W]
            rest = rest.view(B, 2, C, T - 1, H, W).permute(0, 2, 3, 1, 4, 5).reshape(B, C, 2 * (T - 1), H, W)
            x = torch.cat([x[:, :, :1], rest], dim=2)
        x = _frames2d(self.resample, x)
        if self.mode == "downsample3d" and x.shape[2] > 1:
            # frame 0 passes through; a stride-2 temporal conv over [f0, f1, ...] makes the rest
            x = torch.cat([x[:, :, :1], self.time_conv(x)], dim=2)
        return x


class ResidualBlock(nn.Module):
    def __init__(self, in_dim, out_dim):
        super().__init__()
        self.residual = nn.Sequential(RMSNormC(in_dim, images=False), nn.SiLU(),
                                      CausalConv3d(in_dim, out_dim, 3, padding=1),
                                      RMSNormC(out_dim, images=False), nn.SiLU(), nn.Dropout(0.0),
                                      CausalConv3d(out_dim, out_dim, 3, padding=1))
        self.shortcut = CausalConv3d(in_dim, out_dim, 1) if in_dim != out_dim else nn.Identity()

    def forward(self, x):
        return self.residual(x) + self.shortcut(x)


class AttentionBlock(nn.Module):
    """Single-head attention over the pixels of each frame."""

    def __init__(self, dim):
        super().__init__()
        self.norm = RMSNormC(dim)
        self.to_qkv = nn.Conv2d(dim, dim * 3, 1)
        self.proj = nn.Conv2d(dim, dim, 1)
        nn.init.zeros_(self.proj.weight)

    def forward(self, x):
        def per_frame(f):
            n, c, h, w = f.shape
            q, k, v = self.to_qkv(self.norm(f)).reshape(n, 3, c, h * w).transpose(-1, -2).unbind(1)
            o = F.scaled_dot_product_attention(q[:, None], k[:, None], v[:, None])[:, 0]
            return self.proj(o.transpose(-1, -2).reshape(n, c, h, w))
        return x + _frames2d(per_frame, x)


class Encoder3d(nn.Module):
    def __init__(self, dim=96, z_dim=32, dim_mult=(1, 2, 4, 4), num_res_blocks=2, attn_scales=(),
                 temporal_downsample=(False, True, True)):
        super().__init__()
        dims = [dim * u for u in (1,) + tuple(dim_mult)]
        scale = 1.0
        self.conv1 = CausalConv3d(3, dims[0], 3, padding=1)
        layers = []
        for i, (cin, cout) in enumerate(zip(dims[:-1], dims[1:])):
            for _ in range(num_res_blocks):
                layers.append(ResidualBlock(cin, cout))
                if scale in attn_scales:
                    layers.append(AttentionBlock(cout))
                cin = cout
            if i != len(dim_mult) - 1:
                layers.append(Resample(cout, "downsample3d" if temporal_downsample[i] else "downsample2d"))
                scale /= 2.0
        self.downsamples = nn.Sequential(*layers)
        self.middle = nn.Sequential(ResidualBlock(cout, cout), AttentionBlock(cout), ResidualBlock(cout, cout))
        self.head = nn.Sequential(RMSNormC(cout, images=False), nn.SiLU(), CausalConv3d(cout, z_dim, 3, padding=1))

    def forward(self, x):
        return self.head(self.middle(self.downsamples(self.conv1(x))))


class Decoder3d(nn.Module):
    def __init__(self, dim=96, z_dim=16, dim_mult=(1, 2, 4, 4), num_res_blocks=2, attn_scales=(),
                 temporal_upsample=(True, True, False)):
        super().__init__()
        dims = [dim * u for u in (dim_mult[-1],) + tuple(dim_mult[::-1])]
        scale = 1.0 / 2 ** (len(dim_mult) - 2)
        self.conv1 = CausalConv3d(z_dim, dims[0], 3, padding=1)
        self.middle = nn.Sequential(ResidualBlock(dims[0], dims[0]), AttentionBlock(dims[0]),
                                    ResidualBlock(dims[0], dims[0]))
        layers = []
        for i, (cin, cout) in enumerate(zip(dims[:-1], dims[1:])):
            if i in (1, 2, 3):
                cin = cin // 2  # the upsamplers halve the channels
            for _ in range(num_res_blocks + 1):
                layers.append(ResidualBlock(cin, cout))
                if scale in attn_scales:
                    layers.append(AttentionBlock(cout))
                cin = cout
            if i != len(dim_mult) - 1:
                layers.append(Resample(cout, "upsample3d" if temporal_upsample[i] else "upsample2d"))
                scale *= 2.0
        self.upsamples = nn.Sequential(*layers)
        self.head = nn.Sequential(RMSNormC(cout, images=False), nn.SiLU(), CausalConv3d(cout, 3, 3, padding=1))

    def forward(self, x):
        return self.head(self.upsamples(self.middle(self.conv1(x))))


class WanVAEModel(nn.Module):
    """Encoder / decoder pair with the 1x1 causal quant convs (``conv1`` / ``conv2``)."""

    def __init__(self, dim=96, z_dim=16, dim_mult=(1, 2, 4, 4), num_res_blocks=2, attn_scales=(),
                 temporal_downsample=(False, True, True)):
        super().__init__()
        self.z_dim = z_dim
        self.encoder = Encoder3d(dim, z_dim * 2, dim_mult, num_res_blocks, attn_scales, temporal_downsample)
        self.conv1 = CausalConv3d(z_dim * 2, z_dim * 2, 1)
        self.conv2 = CausalConv3d(z_dim, z_dim, 1)
        self.decoder = Decoder3d(dim, z_dim, dim_mult, num_res_blocks, attn_scales, tuple(temporal_downsample[::-1]))


class WanVAE:
    """``encode(video [B, 3, 1+4k, H, W] in [-1, 1]) -> normalised latents [B, 16, 1+k, H/8, W/8]`` and back."""

    def __init__(self, device="cpu", dtype=torch.float32, model: WanVAEModel | None = None):
        self.model = (model or WanVAEModel()).to(device=device, dtype=dtype).eval().requires_grad_(False)
        self.mean = torch.tensor(LATENT_MEAN, device=device, dtype=torch.float32).view(1, -1, 1, 1, 1)
        self.std = torch.tensor(LATENT_STD, device=device, dtype=torch.float32).view(1, -1, 1, 1, 1)
        self.dtype = dtype

    def load_state_dict(self, sd, strict=True):
        return self.model.load_state_dict(sd, strict=strict)

    @staticmethod
    def latent_frames(pixel_frames: int) -> int:
        return 1 + (pixel_frames - 1) // 4

    @staticmethod
    def pixel_frames(latent_frames: int) -> int:
        return (latent_frames - 1) * 4 + 1

    @torch.no_grad()
    def encode(self, video):
        h = self.model.encoder(video.to(self.dtype))
        mu = self.model.conv1(h)[:, : self.model.z_dim].float()
        return (mu - self.mean) / self.std

    @torch.no_grad()
    def decode(self, z):
        z = (z.float() * self.std + self.mean).to(self.dtype)
        return self.model.decoder(self.model.conv2(z)).float().clamp_(-1, 1)
