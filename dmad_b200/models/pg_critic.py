"""Pretrained-feature critic (Projected-GAN style) with two head sets, for the EDM DMAD stack.

Parity: train/image/main/edm/pg_critic.py:24-336 (``PGTwoHeadCritic``), enabled by the critic option
``pretrained_critic="vgg16_bn,tf_efficientnet_lite0"`` (edm_guidance.py:87-91,147-148).  The method is
that of Projected GAN (Sauer et al., NeurIPS 2021): frozen ImageNet feature networks, frozen random
cross-channel (1x1 conv) and cross-scale (top-down fusion with x2 bilinear upsampling) projections,
and trainable spectrally normalised multi-scale conv heads with per-pixel logits and projection class
conditioning.  Two head sets share one feature forward: ``real`` (T vs G) and ``teacher`` (Q vs G).

Feature networks: VGG16-BN from torchvision's architecture, and EfficientNet-Lite0 written here from
its published definition (Tan & Le 2019; the Lite variants drop squeeze-excitation and use ReLU6, with
TensorFlow "same" padding and BatchNorm eps 1e-3).  No weights ship with this repository and nothing is
downloaded: ``load_feature_weights`` reads local state dicts; otherwise the feature networks keep their
random initialisation (a random-feature critic).  The class embedding of every head starts from the
Lite0 classifier weight when that backbone is present, as the reference does.
"""
from __future__ import annotations

import math

import torch
import torch.nn as nn
import torch.nn.functional as F
from torch.nn.utils import spectral_norm

NORMSTATS = {
    "vgg16_bn": {"mean": [0.485, 0.456, 0.406], "std": [0.229, 0.224, 0.225]},
    "tf_efficientnet_lite0": {"mean": [0.5, 0.5, 0.5], "std": [0.5, 0.5, 0.5]},
}


# ----------------------------------------------------------------------------- EfficientNet-Lite0


class _Conv2dSame(nn.Conv2d):
    """Conv with TensorFlow "same" padding: output = ceil(input / stride), extra pad at the end."""

    def forward(self, x):
        ih, iw = x.shape[-2:]
        kh, kw = self.kernel_size
        sh, sw = self.stride
        ph = max((math.ceil(ih / sh) - 1) * sh + kh - ih, 0)
        pw = max((math.ceil(iw / sw) - 1) * sw + kw - iw, 0)
        if ph or pw:
            x = F.pad(x, [pw // 2, pw - pw // 2, ph // 2, ph - ph // 2])
        return F.conv2d(x, self.weight, self.bias, self.stride, 0, self.dilation, self.groups)


def _bn(c):
    return nn.BatchNorm2d(c, eps=1e-3)


class _MBConv(nn.Module):
    """Inverted residual: 1x1 expand (ratio e, skipped for e = 1), kxk depthwise, 1x1 project; ReLU6,
    no squeeze-excitation; identity shortcut when shapes allow."""

    def __init__(self, cin, cout, k, stride, e):
        super().__init__()
        mid = cin * e
        layers = []
        if e != 1:
            layers += [nn.Conv2d(cin, mid, 1, bias=False), _bn(mid), nn.ReLU6(inplace=True)]
        layers += [_Conv2dSame(mid, mid, k, stride, groups=mid, bias=False), _bn(mid), nn.ReLU6(inplace=True),
                   nn.Conv2d(mid, cout, 1, bias=False), _bn(cout)]
        self.body = nn.Sequential(*layers)
        self.residual = stride == 1 and cin == cout

    def forward(self, x):
        y = self.body(x)
        return x + y if self.residual else y


# (expansion, out channels, repeats, stride, kernel) of the seven stages of EfficientNet-B0 / Lite0
_LITE0_STAGES = [(1, 16, 1, 1, 3), (6, 24, 2, 2, 3), (6, 40, 2, 2, 5), (6, 80, 3, 2, 3), (6, 112, 3, 1, 5),
                 (6, 192, 4, 2, 5), (6, 320, 1, 1, 3)]


class EfficientNetLite0(nn.Module):
    def __init__(self, num_classes: int = 1000):
        super().__init__()
        self.conv_stem = _Conv2dSame(3, 32, 3, 2, bias=False)
        self.bn1 = nn.Sequential(_bn(32), nn.ReLU6(inplace=True))
        stages, cin = [], 32
        for e, c, n, s, k in _LITE0_STAGES:
            stages.append(nn.Sequential(*[_MBConv(cin if i == 0 else c, c, k, s if i == 0 else 1, e) for i in range(n)]))
            cin = c
        self.blocks = nn.Sequential(*stages)
        self.conv_head = nn.Conv2d(320, 1280, 1, bias=False)
        self.bn2 = nn.Sequential(_bn(1280), nn.ReLU6(inplace=True))
        self.classifier = nn.Linear(1280, num_classes)

    def forward(self, x):
        x = self.bn2(self.conv_head(self.blocks(self.bn1(self.conv_stem(x)))))
        return self.classifier(x.mean((2, 3)))


# ----------------------------------------------------------------------------- feature networks


def _four_stage(backbone: str):
    """(module with layer0..layer3, lite0 classifier weight or None)."""
    m = nn.Module()
    if backbone == "vgg16_bn":
        import torchvision.models as tvm

        f = tvm.vgg16_bn(weights=None).features
        cuts = [0, 13, 23, 33, 43]  # before pool 2, then through each later block (the reference's split)
        for i in range(4):
            setattr(m, f"layer{i}", nn.Sequential(*list(f)[cuts[i]:cuts[i + 1]]))
        return m, None
    if backbone == "tf_efficientnet_lite0":
        net = EfficientNetLite0()
        m.layer0 = nn.Sequential(net.conv_stem, net.bn1, *net.blocks[0:2])
        m.layer1 = nn.Sequential(*net.blocks[2:3])
        m.layer2 = nn.Sequential(*net.blocks[3:5])
        m.layer3 = nn.Sequential(*net.blocks[5:])
        m.net = net  # keeps the classifier (its weight seeds the class embeddings) and the full state dict
        return m, net.classifier.weight
    raise NotImplementedError(f"feature network {backbone!r} (supported: vgg16_bn, tf_efficientnet_lite0)")


class _Fuse(nn.Module):
    """Cross-scale mixing: add the coarser map, upsample x2 (bilinear, aligned corners), 1x1 conv."""

    def __init__(self, c, expand):
        super().__init__()
        self.out_conv = nn.Conv2d(c, c // 2 if expand else c, 1)

    def forward(self, x, skip=None):
        if skip is not None:
            x = x + skip
        return self.out_conv(F.interpolate(x, scale_factor=2, mode="bilinear", align_corners=True))


class RandomProjFeatures(nn.Module):
    """Frozen feature network + frozen random cross-channel and cross-scale projections; returns the
    four projected maps {"0": finest, ..., "3": coarsest}."""

    def __init__(self, backbone: str, im_res: int = 224, cout: int = 64, expand: bool = True):
        super().__init__()
        self.backbone = backbone
        self.normstats = NORMSTATS[backbone]
        self.pretrained, self._embed = _four_stage(backbone)
        with torch.no_grad():
            t, chans = torch.zeros(1, 3, im_res, im_res), []
            for i in range(4):
                t = getattr(self.pretrained, f"layer{i}")(t)
                chans.append(t.shape[1])
        outs = [cout, cout * 2, cout * 4, cout * 8] if expand else [cout] * 4
        self.ccm = nn.ModuleList([nn.Conv2d(a, b, 1) for a, b in zip(chans, outs)])
        self.csm = nn.ModuleList([_Fuse(outs[0], False), _Fuse(outs[1], expand), _Fuse(outs[2], expand),
                                  _Fuse(outs[3], expand)])
        self.CHANNELS = [cout, cout, cout * 2, cout * 4] if expand else [cout] * 4
        self.RESOLUTIONS = [im_res // 2, im_res // 4, im_res // 8, im_res // 16]

    @property
    def embed_weight(self):
        return None if self._embed is None else self._embed.detach()

    def forward(self, x):
        f, h = [], x
        for i in range(4):
            h = getattr(self.pretrained, f"layer{i}")(h)
            f.append(self.ccm[i](h))
        o3 = self.csm[3](f[3])
        o2 = self.csm[2](o3, f[2])
        o1 = self.csm[1](o2, f[1])
        o0 = self.csm[0](o1, f[0])
        return {"0": o0, "1": o1, "2": o2, "3": o3}


# ----------------------------------------------------------------------------- heads

# channels per resolution of the per-scale heads (the MiDaS table Projected GAN uses)
_NFC = {1: 2048, 2: 1024, 4: 512, 8: 512, 16: 256, 32: 128, 64: 64, 128: 64, 256: 32, 512: 16, 1024: 8}


def _snap(sz):
    return min(_NFC, key=lambda k: abs(k - sz))


class _EqualLinear(nn.Module):
    """Linear with equalised learning rate (weight scaled by 1/sqrt(fan_in) at run time), optionally
    followed by leaky ReLU(0.2) * sqrt(2)."""

    def __init__(self, fin, fout, lrelu=False):
        super().__init__()
        self.weight = nn.Parameter(torch.randn(fout, fin))
        self.bias = nn.Parameter(torch.zeros(fout))
        self.gain = 1.0 / math.sqrt(fin)
        self.lrelu = lrelu

    def forward(self, x):
        y = F.linear(x, self.weight * self.gain, self.bias)
        return F.leaky_relu(y, 0.2) * math.sqrt(2) if self.lrelu else y


class _ScaleHead(nn.Module):
    """Strided SN convs down to ``end_sz``, an SN conv to ``cmap_dim`` channels, and the projection onto
    the class embedding: per-pixel logits [N, 1, h, w]."""

    def __init__(self, nc, start_sz, end_sz=8, c_dim=1000, cmap_dim=64, embed_weight=None):
        super().__init__()
        sz = _snap(start_sz)
        nfc = dict(_NFC)
        nfc[sz] = nc
        layers = []
        while sz > end_sz:
            layers += [spectral_norm(nn.Conv2d(nfc[sz], nfc[sz // 2], 4, 2, 1)), nn.BatchNorm2d(nfc[sz // 2]),
                       nn.LeakyReLU(0.2, inplace=True)]
            sz //= 2
        self.main = nn.Sequential(*layers)
        k = 4 if end_sz >= 8 else max(1, end_sz // 2)
        self.cls = spectral_norm(nn.Conv2d(nfc[end_sz], cmap_dim, k, 1, 0, bias=False))
        self.embed = (nn.Embedding.from_pretrained(embed_weight.clone(), freeze=False) if embed_weight is not None
                      else nn.Embedding(c_dim, 320))
        self.embed_proj = _EqualLinear(self.embed.embedding_dim, cmap_dim, lrelu=True)
        self.cmap_dim = cmap_dim

    def forward(self, x, c_onehot):
        out = self.cls(self.main(x))
        cmap = self.embed_proj(self.embed(c_onehot.argmax(1)))[:, :, None, None]
        return (out * cmap).sum(1, keepdim=True) / math.sqrt(self.cmap_dim)


class _MultiScaleHeads(nn.Module):
    def __init__(self, channels, resolutions, c_dim, embed_weight):
        super().__init__()
        end = 8 if resolutions[-1] >= 8 else resolutions[-1]
        self.heads = nn.ModuleList([_ScaleHead(c, r, end, c_dim, embed_weight=embed_weight)
                                    for c, r in zip(channels, resolutions)])

    def forward(self, feats, c):
        return torch.cat([h(feats[str(i)], c).flatten(1) for i, h in enumerate(self.heads)], dim=1)


class PGTwoHeadCritic(nn.Module):
    """``forward(x in [-1, 1], one-hot labels) -> (d_real [N, K], d_teacher [N, K])``: per-pixel logits of
    every head of every feature network; no noise-level input."""

    def __init__(self, backbones=("vgg16_bn", "tf_efficientnet_lite0"), c_dim: int = 1000, im_res: int = 224):
        super().__init__()
        self.im_res = im_res
        self.features = nn.ModuleDict({b: RandomProjFeatures(b, im_res) for b in backbones})
        embed = next((f.embed_weight for f in self.features.values() if f.embed_weight is not None), None)
        self.heads_real = nn.ModuleDict({b: _MultiScaleHeads(f.CHANNELS, f.RESOLUTIONS, c_dim, embed)
                                         for b, f in self.features.items()})
        self.heads_teacher = nn.ModuleDict({b: _MultiScaleHeads(f.CHANNELS, f.RESOLUTIONS, c_dim, embed)
                                            for b, f in self.features.items()})
        self.features.requires_grad_(False)

    def train(self, mode: bool = True):
        super().train(mode)
        self.features.train(False)  # frozen networks (and their BatchNorms) always in eval mode
        return self

    def load_feature_weights(self, backbone: str, state_dict: dict, strict: bool = True):
        """Loads a local state dict of the full feature network (torchvision ``vgg16_bn().features``
        keys for VGG, this module's ``EfficientNetLite0`` keys for Lite0)."""
        f = self.features[backbone].pretrained
        if backbone == "vgg16_bn":
            seq = nn.Sequential(*[m for i in range(4) for m in getattr(f, f"layer{i}")])
            sd = {k[len("features."):] if k.startswith("features.") else k: v for k, v in state_dict.items()}
            sd = {k: v for k, v in sd.items() if int(k.split(".")[0]) < len(seq)}
            return seq.load_state_dict(sd, strict=strict)
        return f.net.load_state_dict(state_dict, strict=strict)

    def _inputs(self, x, feat):
        x = (x.float() + 1) / 2
        mean = x.new_tensor(feat.normstats["mean"]).view(1, 3, 1, 1)
        std = x.new_tensor(feat.normstats["std"]).view(1, 3, 1, 1)
        return F.interpolate((x - mean) / std, self.im_res, mode="bilinear", align_corners=False)

    def forward(self, x, c):
        d_r, d_t = [], []
        for b, feat in self.features.items():
            fm = feat(self._inputs(x, feat))
            d_r.append(self.heads_real[b](fm, c))
            d_t.append(self.heads_teacher[b](fm, c))
        return torch.cat(d_r, dim=1), torch.cat(d_t, dim=1)
