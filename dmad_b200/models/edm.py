"""EDM-preconditioned ADM-style U-Net for the class-conditional image path.

Parity with train/image/third_party/edm/training/networks.py:
* ``EDMPrecond`` (:638-686): c_skip = s_d^2/(s^2+s_d^2), c_out = s s_d / sqrt(s^2+s_d^2),
  c_in = 1/sqrt(s_d^2+s^2), c_noise = log(s)/4; bf16 body when ``use_fp16`` on CUDA;
* ``DhariwalUNet`` (:373-467): positional noise embedding -> 2 Linears (SiLU) + label embedding;
  encoder ``{res}x{res}_conv`` / ``_down`` / ``_block{i}`` and decoder ``_in0`` / ``_in1`` / ``_up`` /
  ``_block{i}`` with skip concatenation; ``return_bottleneck`` returns the encoder output;
* ``UNetBlock`` (:133-192): GroupNorm-SiLU-conv, adaptive scale/shift from the embedding, residual
  skip (1x1 conv when channels change), optional multi-head self-attention (64 channels per head);
  up/down sampling with the [1, 1] resample filter (2x2 box average / nearest-neighbour).
Module names follow the reference, so the two state dicts line up.
"""
from __future__ import annotations

import math

import numpy as np
import torch
import torch.nn as nn
import torch.nn.functional as F


class PositionalEmbedding(nn.Module):
    def __init__(self, num_channels, max_positions=10000, endpoint=False):
        super().__init__()
        self.num_channels, self.max_positions, self.endpoint = num_channels, max_positions, endpoint

    def forward(self, x):
        half = self.num_channels // 2
        freqs = torch.arange(half, dtype=torch.float32, device=x.device) / (half - (1 if self.endpoint else 0))
        freqs = (1 / self.max_positions) ** freqs
        x = x.float().ger(freqs)
        return torch.cat([x.cos(), x.sin()], dim=1)


def _gn(c, eps=1e-5):
    return nn.GroupNorm(min(32, c // 4), c, eps=eps)


class UNetBlock(nn.Module):
    def __init__(self, in_channels, out_channels, emb_channels, up=False, down=False, attention=False,
                 channels_per_head=64, dropout=0.0, eps=1e-5):
        super().__init__()
        self.in_channels, self.out_channels = in_channels, out_channels
        self.up, self.down, self.dropout = up, down, dropout
        self.num_heads = out_channels // channels_per_head if attention else 0
        self.norm0 = _gn(in_channels, eps)
        self.conv0 = nn.Conv2d(in_channels, out_channels, 3, padding=1)
        self.affine = nn.Linear(emb_channels, out_channels * 2)
        self.norm1 = _gn(out_channels, eps)
        self.conv1 = nn.Conv2d(out_channels, out_channels, 3, padding=1)
        self.skip = None
        if out_channels != in_channels or up or down:
            self.skip = nn.Conv2d(in_channels, out_channels, 1) if out_channels != in_channels else nn.Identity()
        if self.num_heads:
            self.norm2 = _gn(out_channels, eps)
            self.qkv = nn.Conv2d(out_channels, out_channels * 3, 1)
            self.proj = nn.Conv2d(out_channels, out_channels, 1)
            nn.init.zeros_(self.proj.weight)
            nn.init.zeros_(self.proj.bias)
        nn.init.zeros_(self.conv1.weight)
        nn.init.zeros_(self.conv1.bias)

    def _resample(self, x):
        if self.up:
            return F.interpolate(x, scale_factor=2, mode="nearest")
        if self.down:
            return F.avg_pool2d(x, 2)
        return x

    def forward(self, x, emb):
        orig = x
        x = self.conv0(self._resample(F.silu(self.norm0(x))))
        scale, shift = self.affine(emb).unsqueeze(2).unsqueeze(3).to(x.dtype).chunk(2, dim=1)
        x = F.silu(torch.addcmul(shift, self.norm1(x), scale + 1))
        x = self.conv1(F.dropout(x, p=self.dropout, training=self.training))
        res = orig
        if self.skip is not None:
            res = self.skip(self._resample(orig))
        x = x + res
        if self.num_heads:
            B, C, H, W = x.shape
            q, k, v = self.qkv(self.norm2(x)).reshape(B, self.num_heads, C // self.num_heads, 3, H * W).unbind(3)
            a = F.scaled_dot_product_attention(q.transpose(-1, -2).float(), k.transpose(-1, -2).float(),
                                               v.transpose(-1, -2).float()).to(x.dtype)
            x = self.proj(a.transpose(-1, -2).reshape(B, C, H, W)) + x
        return x


class DhariwalUNet(nn.Module):
    def __init__(self, img_resolution, in_channels, out_channels, label_dim=0, model_channels=192,
                 channel_mult=(1, 2, 3, 4), channel_mult_emb=4, num_blocks=3, attn_resolutions=(32, 16, 8),
                 dropout=0.0):
        super().__init__()
        emb = model_channels * channel_mult_emb
        bk = dict(emb_channels=emb, channels_per_head=64, dropout=dropout)
        self.map_noise = PositionalEmbedding(model_channels)
        self.map_layer0 = nn.Linear(model_channels, emb)
        self.map_layer1 = nn.Linear(emb, emb)
        self.map_label = nn.Linear(label_dim, emb, bias=False) if label_dim else None
        if self.map_label is not None:
            nn.init.normal_(self.map_label.weight, std=1.0)
        self.enc = nn.ModuleDict()
        cout = in_channels
        for level, mult in enumerate(channel_mult):
            res = img_resolution >> level
            if level == 0:
                cin, cout = cout, model_channels * mult
                self.enc[f"{res}x{res}_conv"] = nn.Conv2d(cin, cout, 3, padding=1)
            else:
                self.enc[f"{res}x{res}_down"] = UNetBlock(cout, cout, down=True, **bk)
            for i in range(num_blocks):
                cin, cout = cout, model_channels * mult
                self.enc[f"{res}x{res}_block{i}"] = UNetBlock(cin, cout, attention=res in attn_resolutions, **bk)
        skips = [b.out_channels if isinstance(b, UNetBlock) else b.out_channels for b in self.enc.values()]
        self.bottleneck_channels = cout
        self.dec = nn.ModuleDict()
        for level, mult in reversed(list(enumerate(channel_mult))):
            res = img_resolution >> level
            if level == len(channel_mult) - 1:
                self.dec[f"{res}x{res}_in0"] = UNetBlock(cout, cout, attention=True, **bk)
                self.dec[f"{res}x{res}_in1"] = UNetBlock(cout, cout, **bk)
            else:
                self.dec[f"{res}x{res}_up"] = UNetBlock(cout, cout, up=True, **bk)
            for i in range(num_blocks + 1):
                cin, cout = cout + skips.pop(), model_channels * mult
                self.dec[f"{res}x{res}_block{i}"] = UNetBlock(cin, cout, attention=res in attn_resolutions, **bk)
        self.out_norm = _gn(cout)
        self.out_conv = nn.Conv2d(cout, out_channels, 3, padding=1)
        nn.init.zeros_(self.out_conv.weight)
        nn.init.zeros_(self.out_conv.bias)

    def forward(self, x, noise_labels, class_labels, return_bottleneck=False):
        emb = F.silu(self.map_layer0(self.map_noise(noise_labels)))
        emb = self.map_layer1(emb)
        if self.map_label is not None:
            emb = emb + self.map_label(class_labels)
        emb = F.silu(emb).to(x.dtype)
        skips = []
        for blk in self.enc.values():
            x = blk(x, emb) if isinstance(blk, UNetBlock) else blk(x)
            skips.append(x)
        if return_bottleneck:
            return x
        for blk in self.dec.values():
            if x.shape[1] != blk.in_channels:
                x = torch.cat([x, skips.pop()], dim=1)
            x = blk(x, emb)
        return self.out_conv(F.silu(self.out_norm(x)))


class EDMPrecond(nn.Module):
    def __init__(self, img_resolution, img_channels, label_dim=0, use_fp16=False, sigma_data=0.5, **unet_kwargs):
        super().__init__()
        self.img_resolution, self.img_channels, self.label_dim = img_resolution, img_channels, label_dim
        self.use_fp16, self.sigma_data = use_fp16, sigma_data
        self.model = DhariwalUNet(img_resolution, img_channels, img_channels, label_dim=label_dim, **unet_kwargs)

    def forward(self, x, sigma, class_labels=None, return_bottleneck=False):
        x = x.float()
        sigma = sigma.float().reshape(-1, 1, 1, 1)
        sd = self.sigma_data
        c_skip = sd ** 2 / (sigma ** 2 + sd ** 2)
        c_out = sigma * sd / (sigma ** 2 + sd ** 2).sqrt()
        c_in = 1 / (sd ** 2 + sigma ** 2).sqrt()
        c_noise = sigma.log() / 4
        dtype = torch.bfloat16 if (self.use_fp16 and x.is_cuda) else torch.float32
        labels = None if self.label_dim == 0 else class_labels.float().reshape(-1, self.label_dim)
        Fx = self.model((c_in * x).to(dtype), c_noise.flatten(), labels, return_bottleneck=return_bottleneck)
        if return_bottleneck:
            return Fx
        return c_skip * x + c_out * Fx.float()


def config1_unet(label_dim=1000):
    """64x64x3, base channels 64, mult [1, 2, 2], 1 block per level, attention at 16x16."""
    return EDMPrecond(64, 3, label_dim=label_dim, model_channels=64, channel_mult=(1, 2, 2), channel_mult_emb=4,
                      num_blocks=1, attn_resolutions=(16,))


def imagenet_unet(label_dim=1000, use_fp16=False):
    """The reference's ImageNet-64 configuration (train/image/main/edm/edm_network.py:3-31)."""
    return EDMPrecond(64, 3, label_dim=label_dim, use_fp16=use_fp16, model_channels=192, channel_mult=(1, 2, 3, 4),
                      channel_mult_emb=4, num_blocks=3, attn_resolutions=(32, 16, 8))


# ----------------------------------------------------------------------------- pretrained teachers


class _Record:
    """Stands in for a class of a pickled network: keeps the instance's attribute dict, runs nothing."""

    def __init__(self, *args, **kwargs):
        pass

    def __setstate__(self, state):
        if isinstance(state, tuple):  # (dict, slots) form
            state = state[0] or {}
        if isinstance(state, dict):
            self.__dict__.update(state)


def _persistent_record(meta):
    """An EDM ``torch_utils.persistence`` record: the object's state is kept, its embedded module source
    is never executed."""
    obj = _Record()
    obj.__setstate__(meta.get("state", {}) if isinstance(meta, dict) else {})
    return obj


def _storage_from_bytes(b):
    """A tensor storage serialised inside a plain pickle, read with torch's weights-only loader."""
    import io

    return torch.load(io.BytesIO(b), weights_only=True)


_TORCH_REBUILD = {"_rebuild_tensor_v2", "_rebuild_parameter", "_rebuild_parameter_with_state"}
_PLAIN = {("collections", "OrderedDict"), ("builtins", "set"), ("builtins", "frozenset")}


def _net_unpickler(f):
    """A ``pickle.Unpickler`` that rebuilds tensors and containers but replaces every other class by
    ``_Record``: no code of the pickle runs (torch's tensor rebuild functions, a weights-only storage
    loader, ``OrderedDict`` and plain builtin containers are the only callables it resolves)."""
    import pickle

    class Unpickler(pickle.Unpickler):
        def find_class(self, module, name):
            if module == "torch._utils" and name in _TORCH_REBUILD:
                return super().find_class(module, name)
            if (module, name) in _PLAIN:
                return super().find_class(module, name)
            if (module, name) == ("torch.storage", "_load_from_bytes"):
                return _storage_from_bytes
            if module.endswith("persistence") and name == "_reconstruct_persistent_obj":
                return _persistent_record
            if (module, name) == ("copyreg", "_reconstructor"):
                return lambda *a: _Record()
            return type(name, (_Record,), {})

        def persistent_load(self, pid):
            raise pickle.UnpicklingError("persistent ids are not supported")

    return Unpickler(f)


def _record_state_dict(obj, prefix="", out=None):
    """``state_dict`` of a module rebuilt from ``_Record`` objects: its ``_parameters`` / ``_buffers`` /
    ``_modules`` attribute dicts, walked recursively (non-persistent buffers skipped)."""
    out = {} if out is None else out
    d = obj.__dict__ if not isinstance(obj, nn.Module) else {
        "_parameters": obj._parameters, "_buffers": obj._buffers, "_modules": obj._modules,
        "_non_persistent_buffers_set": obj._non_persistent_buffers_set}
    skip = d.get("_non_persistent_buffers_set") or set()
    for k, v in (d.get("_parameters") or {}).items():
        if v is not None:
            out[prefix + k] = v.detach()
    for k, v in (d.get("_buffers") or {}).items():
        if v is not None and k not in skip:
            out[prefix + k] = v
    for k, v in (d.get("_modules") or {}).items():
        if v is not None:
            _record_state_dict(v, f"{prefix}{k}.", out)
    return out


def read_edm_teacher(path: str) -> dict:
    """The state dict of a pretrained EDM network.

    ``.pkl``: an EDM release pickle (its ``"ema"`` entry), read with ``_net_unpickler``, so neither the
    EDM code nor the source embedded in the pickle is needed or run (the reference unpickles it with the
    EDM code importable: train/image/main/edm/edm_unified_model.py:13-21).  ``.safetensors`` or a torch
    file: a state dict (an ``"ema"`` / ``"model"`` / ``"state_dict"`` entry is unwrapped)."""
    if path.endswith(".pkl"):
        with open(path, "rb") as f:
            data = _net_unpickler(f).load()
        return _record_state_dict(data["ema"] if isinstance(data, dict) else data)
    if path.endswith(".safetensors"):
        from safetensors.torch import load_file
        return load_file(path)
    sd = torch.load(path, map_location="cpu", weights_only=True)
    for key in ("ema", "model", "state_dict"):
        if isinstance(sd, dict) and isinstance(sd.get(key), dict):
            sd = sd[key]
    return sd


def load_edm_teacher(net: "EDMPrecond", path: str) -> "EDMPrecond":
    """Loads a pretrained EDM teacher into ``net``: every key must match, except the augmentation
    mapping, which the distillation drops (edm_unified_model.py:18-20)."""
    sd = {k: v for k, v in read_edm_teacher(path).items() if ".map_augment." not in k}
    res = net.load_state_dict(sd, strict=False)
    if res.missing_keys or res.unexpected_keys:
        raise KeyError(f"EDM teacher {path}: missing {res.missing_keys[:3]}, unexpected {res.unexpected_keys[:3]}")
    return net
