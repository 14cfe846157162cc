"""SDXL-shaped conditional U-Net: the architecture of the SDXL base UNet
(diffusers ``UNet2DConditionModel`` as loaded by train/image/main/sd_guidance.py and
sd_unified_model.py), written from its published structure:

* ``conv_in`` 4 -> 320; timestep sinusoid (320) -> ``time_embedding`` 320 -> 1280 -> 1280;
  ``add_embedding``: [sinusoid(256) of the 6 size/crop ids ; pooled text 1280] (2816) -> 1280 -> 1280;
* down: (320, 2 ResNets, no attention, downsample), (640, 2 ResNets, 2 transformers of depth 2,
  downsample), (1280, 2 ResNets, 2 transformers of depth 10); mid: ResNet, transformer of depth 10,
  ResNet; up: mirrored with 3 ResNets per level; GroupNorm(32) + SiLU + ``conv_out`` 320 -> 4;
* transformers: GroupNorm -> Linear in -> [LN, self-attn; LN, cross-attn to the 77 x 2048 text;
  LN, GEGLU feed-forward x4] x depth -> Linear out, residual; heads of 64 channels (on CUDA the
  tcgen05 flash kernels, forward and backward; on the CPU PyTorch's SDPA).
``classify_forward`` (train/image/main/sd_unet_forward.py) = encoder + mid block only, returning the
bottleneck (``return_bottleneck=True``).  Random-init weights; ~2.6 B parameters.
"""
from __future__ import annotations

import math

import torch
import torch.nn as nn
import torch.nn.functional as F
from torch.utils.checkpoint import checkpoint


def timestep_sinusoid(t, dim, flip_sin_to_cos=True, shift=0.0, max_period=10000):
    half = dim // 2
    exponent = -math.log(max_period) * torch.arange(half, dtype=torch.float32, device=t.device) / (half - shift)
    emb = t.float()[:, None] * torch.exp(exponent)[None]
    emb = torch.cat([torch.sin(emb), torch.cos(emb)], dim=-1)
    return torch.cat([emb[:, half:], emb[:, :half]], dim=-1) if flip_sin_to_cos else emb


class ResnetBlock(nn.Module):
    def __init__(self, cin, cout, temb=1280):
        super().__init__()
        self.norm1 = nn.GroupNorm(32, cin, eps=1e-5)
        self.conv1 = nn.Conv2d(cin, cout, 3, padding=1)
        self.time_emb_proj = nn.Linear(temb, cout)
        self.norm2 = nn.GroupNorm(32, cout, eps=1e-5)
        self.conv2 = nn.Conv2d(cout, cout, 3, padding=1)
        self.conv_shortcut = nn.Conv2d(cin, cout, 1) if cin != cout else None

    def forward(self, x, temb):
        h = self.conv1(F.silu(self.norm1(x)))
        h = h + self.time_emb_proj(F.silu(temb))[:, :, None, None].to(h.dtype)
        h = self.conv2(F.silu(self.norm2(h)))
        return h + (self.conv_shortcut(x) if self.conv_shortcut is not None else x)


class Attention(nn.Module):
    def __init__(self, dim, ctx_dim=None, head_dim=64):
        super().__init__()
        self.heads = dim // head_dim
        self.to_q = nn.Linear(dim, dim, bias=False)
        self.to_k = nn.Linear(ctx_dim or dim, dim, bias=False)
        self.to_v = nn.Linear(ctx_dim or dim, dim, bias=False)
        self.to_out = nn.ModuleList([nn.Linear(dim, dim)])

    def forward(self, x, ctx=None):
        ctx = x if ctx is None else ctx
        B, N, C = x.shape
        q = self.to_q(x).view(B, N, self.heads, -1)
        k = self.to_k(ctx).view(B, ctx.shape[1], self.heads, -1)
        v = self.to_v(ctx).view(B, ctx.shape[1], self.heads, -1)
        if x.is_cuda:  # the tcgen05 flash kernels (head dim 64), forward and backward
            from .. import ops
            o = ops.flash_attention(q, k, v)
        else:
            o = F.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2)).transpose(1, 2)
        return self.to_out[0](o.reshape(B, N, C))


class GEGLU(nn.Module):
    def __init__(self, dim, inner):
        super().__init__()
        self.proj = nn.Linear(dim, inner * 2)

    def forward(self, x):
        h, g = self.proj(x).chunk(2, dim=-1)
        return h * F.gelu(g)


class BasicTransformerBlock(nn.Module):
    def __init__(self, dim, ctx_dim):
        super().__init__()
        self.norm1 = nn.LayerNorm(dim)
        self.attn1 = Attention(dim)
        self.norm2 = nn.LayerNorm(dim)
        self.attn2 = Attention(dim, ctx_dim)
        self.norm3 = nn.LayerNorm(dim)
        self.ff = nn.Module()
        self.ff.net = nn.ModuleList([GEGLU(dim, 4 * dim), nn.Dropout(0.0), nn.Linear(4 * dim, dim)])

    def forward(self, x, ctx):
        x = x + self.attn1(self.norm1(x))
        x = x + self.attn2(self.norm2(x), ctx)
        h = self.norm3(x)
        for m in self.ff.net:
            h = m(h)
        return x + h


class Transformer2D(nn.Module):
    def __init__(self, ch, depth, ctx_dim):
        super().__init__()
        self.norm = nn.GroupNorm(32, ch, eps=1e-6)
        self.proj_in = nn.Linear(ch, ch)
        self.transformer_blocks = nn.ModuleList([BasicTransformerBlock(ch, ctx_dim) for _ in range(depth)])
        self.proj_out = nn.Linear(ch, ch)

    def forward(self, x, ctx):
        B, C, H, W = x.shape
        h = self.norm(x).permute(0, 2, 3, 1).reshape(B, H * W, C)
        h = self.proj_in(h)
        for blk in self.transformer_blocks:
            h = blk(h, ctx)
        h = self.proj_out(h).reshape(B, H, W, C).permute(0, 3, 1, 2)
        return h + x


class _Level(nn.Module):
    def __init__(self, resnets, attentions, sampler=None, sampler_name=None):
        super().__init__()
        self.resnets = nn.ModuleList(resnets)
        self.attentions = nn.ModuleList(attentions) if attentions else None
        if sampler is not None:
            setattr(self, sampler_name, nn.ModuleList([sampler]))
        self.sampler_name = sampler_name


class _Down(nn.Module):
    def __init__(self, ch):
        super().__init__()
        self.conv = nn.Conv2d(ch, ch, 3, stride=2, padding=1)

    def forward(self, x):
        return self.conv(x)


class _Up(nn.Module):
    def __init__(self, ch):
        super().__init__()
        self.conv = nn.Conv2d(ch, ch, 3, padding=1)

    def forward(self, x):
        return self.conv(F.interpolate(x, scale_factor=2.0, mode="nearest"))


class SDXLUNet(nn.Module):
    def __init__(self, in_channels=4, channels=(320, 640, 1280), depths=(0, 2, 10), ctx_dim=2048, pooled_dim=1280,
                 addition_time_embed_dim=256, layers_per_block=2):
        super().__init__()
        c0 = channels[0]
        temb = c0 * 4
        self.channels, self.depths = channels, depths
        self.addition_time_embed_dim = addition_time_embed_dim
        self.conv_in = nn.Conv2d(in_channels, c0, 3, padding=1)
        self.time_embedding = nn.Module()
        self.time_embedding.linear_1 = nn.Linear(c0, temb)
        self.time_embedding.linear_2 = nn.Linear(temb, temb)
        self.add_embedding = nn.Module()
        self.add_embedding.linear_1 = nn.Linear(6 * addition_time_embed_dim + pooled_dim, temb)
        self.add_embedding.linear_2 = nn.Linear(temb, temb)
        self.down_blocks = nn.ModuleList()
        skip_ch = [c0]
        cin = c0
        for i, (ch, d) in enumerate(zip(channels, depths)):
            res, att = [], []
            for _ in range(layers_per_block):
                res.append(ResnetBlock(cin, ch, temb))
                if d:
                    att.append(Transformer2D(ch, d, ctx_dim))
                cin = ch
                skip_ch.append(ch)
            last = i == len(channels) - 1
            self.down_blocks.append(_Level(res, att, None if last else _Down(ch), None if last else "downsamplers"))
            if not last:
                skip_ch.append(ch)
        self.mid_block = nn.Module()
        self.mid_block.resnets = nn.ModuleList([ResnetBlock(cin, cin, temb), ResnetBlock(cin, cin, temb)])
        self.mid_block.attentions = nn.ModuleList([Transformer2D(cin, depths[-1], ctx_dim)])
        self.up_blocks = nn.ModuleList()
        for i, (ch, d) in enumerate(zip(reversed(channels), reversed(depths))):
            res, att = [], []
            for _ in range(layers_per_block + 1):
                res.append(ResnetBlock(cin + skip_ch.pop(), ch, temb))
                if d:
                    att.append(Transformer2D(ch, d, ctx_dim))
                cin = ch
            last = i == len(channels) - 1
            self.up_blocks.append(_Level(res, att, None if last else _Up(ch), None if last else "upsamplers"))
        self.conv_norm_out = nn.GroupNorm(32, c0, eps=1e-5)
        self.conv_out = nn.Conv2d(c0, in_channels, 3, padding=1)
        self.gradient_checkpointing = False

    def embed(self, t, time_ids, pooled):
        te = timestep_sinusoid(t, self.channels[0])
        emb = self.time_embedding.linear_2(F.silu(self.time_embedding.linear_1(te.to(self.conv_in.weight.dtype))))
        ids = timestep_sinusoid(time_ids.reshape(-1), self.addition_time_embed_dim).reshape(time_ids.shape[0], -1)
        add = torch.cat([pooled, ids.to(pooled.dtype)], dim=-1).to(emb.dtype)
        return emb + self.add_embedding.linear_2(F.silu(self.add_embedding.linear_1(add)))

    def _run(self, m, *a):
        if self.gradient_checkpointing and self.training and torch.is_grad_enabled():
            return checkpoint(m, *a, use_reentrant=False)
        return m(*a)

    def forward(self, x, t, ctx, time_ids, pooled, return_bottleneck=False):
        emb = self.embed(t, time_ids, pooled)
        h = self.conv_in(x)
        skips = [h]
        for lvl in self.down_blocks:
            for i, r in enumerate(lvl.resnets):
                h = self._run(r, h, emb)
                if lvl.attentions is not None:
                    h = self._run(lvl.attentions[i], h, ctx)
                skips.append(h)
            if lvl.sampler_name:
                h = getattr(lvl, lvl.sampler_name)[0](h)
                skips.append(h)
        h = self._run(self.mid_block.resnets[0], h, emb)
        h = self._run(self.mid_block.attentions[0], h, ctx)
        h = self._run(self.mid_block.resnets[1], h, emb)
        if return_bottleneck:
            return h
        for lvl in self.up_blocks:
            for i, r in enumerate(lvl.resnets):
                h = self._run(r, torch.cat([h, skips.pop()], dim=1), emb)
                if lvl.attentions is not None:
                    h = self._run(lvl.attentions[i], h, ctx)
            if lvl.sampler_name:
                h = getattr(lvl, lvl.sampler_name)[0](h)
        return self.conv_out(F.silu(self.conv_norm_out(h)))


def ddpm_alphas_cumprod(n=1000, beta_start=0.00085, beta_end=0.012):
    """SDXL's scaled-linear schedule."""
    betas = torch.linspace(beta_start ** 0.5, beta_end ** 0.5, n, dtype=torch.float64) ** 2
    return torch.cumprod(1.0 - betas, dim=0)
