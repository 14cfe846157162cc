"""Frozen-gain spectral normalisation of plain layers (``nn.Linear``, ``nn.Conv1d/2d/3d``).

The effective weight is ``W * g / sigma(W)``: ``sigma(W)`` is the largest singular value of the weight
(flattened to ``[out, in * k...]``), estimated by power iteration with a persistent left / right vector
pair, and ``g`` is ``sigma`` measured once at set-up and frozen, so the layer computes exactly what it
computed before normalisation and afterwards its spectral norm stays at its initial value while ``W``
trains.  This is the normalisation the reference registers on its critics (train/wan/rcm/models/
t2v_model_distill_dmad.py:488-517, train/image/main/edm/edm_guidance.py:54-80,
train/image/main/sd_guidance.py:51-89); the power method is Miyato et al. 2018 ("Spectral
Normalization for GANs").  The fused projections of the DiTs carry the same normalisation inside
``SegLinear`` (``models/layers.py``); this module covers every other layer.

Design: the layer's class is switched to a subclass whose ``forward`` applies the normalised weight;
the parameter stays ``weight`` and the state is three buffers ``sn_u`` / ``sn_v`` / ``sn_gain`` (the key
names ``SegLinear`` and the reference-checkpoint importer use), so modules deep-copy, pickle and load
state dicts like any other.  ``update`` selects when a power step runs: ``"train"`` (in training mode
only, the Wan / EDM critics) or ``"always"`` (every forward, the SDXL critic).
"""
from __future__ import annotations

import torch
import torch.nn as nn
import torch.nn.functional as F


def _unit(x: torch.Tensor, eps: float = 1e-12) -> torch.Tensor:
    return x / x.norm().clamp_min(eps)


def power_iterate(mat: torch.Tensor, u: torch.Tensor, iters: int) -> tuple[torch.Tensor, torch.Tensor]:
    """``iters`` steps v <- W^T u / |.|, u <- W v / |.| from ``u``; returns (u, v)."""
    v = _unit(mat.t() @ u)
    for _ in range(iters):
        v = _unit(mat.t() @ u)
        u = _unit(mat @ v)
    return u, v


class _SpectralWeight:
    """Mixin: the normalised weight, one power step first when the update rule says so."""

    sn_update: str = "train"

    def sn_weight(self) -> torch.Tensor:
        w = self.weight
        mat = w.flatten(1).float()
        if self.sn_update == "always" or self.training:
            with torch.no_grad():
                v = _unit(mat.t() @ self.sn_u.float())
                u = _unit(mat @ v)
                self.sn_u.copy_(u)
                self.sn_v.copy_(v)
        # copies: a later forward updates the buffers in place while this graph still needs them
        u = self.sn_u.float().clone()
        v = self.sn_v.float().clone()
        sigma = torch.dot(u, mat @ v)
        return (w.float() * (self.sn_gain.float() / sigma)).to(w.dtype)


class SNLinear(_SpectralWeight, nn.Linear):
    def forward(self, x):
        return F.linear(x, self.sn_weight(), self.bias)


class SNConv1d(_SpectralWeight, nn.Conv1d):
    def forward(self, x):
        return self._conv_forward(x, self.sn_weight(), self.bias)


class SNConv2d(_SpectralWeight, nn.Conv2d):
    def forward(self, x):
        return self._conv_forward(x, self.sn_weight(), self.bias)


class SNConv3d(_SpectralWeight, nn.Conv3d):
    def forward(self, x):
        return self._conv_forward(x, self.sn_weight(), self.bias)


_SN_CLASS = {nn.Linear: SNLinear, nn.Conv1d: SNConv1d, nn.Conv2d: SNConv2d, nn.Conv3d: SNConv3d}


@torch.no_grad()
def attach_spectral_norm(layer: nn.Module, power_iters: int = 30, update: str = "train",
                         allow_frozen: bool = False, seed: int | None = None) -> bool:
    """Puts the frozen-gain spectral norm on one layer; returns whether it did.

    Skipped (False): a layer that is not a plain Linear / Conv, one already normalised, a frozen weight
    unless ``allow_frozen``, and a weight whose spectral norm is ~0 (a zero-initialised output layer:
    sigma would divide by zero), as the reference skips them."""
    cls = _SN_CLASS.get(type(layer))
    if cls is None:
        return False
    w = layer.weight
    if not isinstance(w, nn.Parameter) or w.dim() < 2 or (not w.requires_grad and not allow_frozen):
        return False
    mat = w.detach().flatten(1).float()
    assert update in ("train", "always"), update
    gen = torch.Generator(device="cpu")
    gen.manual_seed(seed if seed is not None else 0x5EC7)
    u0 = _unit(torch.randn(mat.shape[0], generator=gen).to(mat.device))
    u, v = power_iterate(mat, u0, max(1, int(power_iters)))
    sigma0 = torch.dot(u, mat @ v)
    if float(sigma0) < 1e-8:  # the power-iteration estimate of the spectral norm (no SVD)
        return False
    layer.register_buffer("sn_u", u.to(w.dtype if w.dtype.is_floating_point else torch.float32))
    layer.register_buffer("sn_v", v.to(layer.sn_u.dtype))
    layer.register_buffer("sn_gain", sigma0.reshape(()).to(torch.float32))
    layer.__class__ = cls
    layer.sn_update = update
    return True


def apply_spectral_norm(module: nn.Module, power_iters: int = 30, update: str = "train",
                        types: tuple = (nn.Linear, nn.Conv1d, nn.Conv2d, nn.Conv3d), allow_frozen: bool = False) -> int:
    """``attach_spectral_norm`` on every sub-layer of ``module`` of one of ``types``; returns the count."""
    n = 0
    for m in list(module.modules()):
        if type(m) in _SN_CLASS and issubclass(type(m), types):
            n += attach_spectral_norm(m, power_iters, update, allow_frozen, seed=n)
    return n


@torch.no_grad()
def fold_spectral_norm(module: nn.Module) -> int:
    """Replaces every normalised layer's weight by the effective weight its forward would use in the
    layer's current mode (in eval mode a ``"train"`` layer takes no power step) and turns the layer back
    into its plain class, so the plain network reproduces the normalised one; returns the count."""
    n = 0
    inverse = {v: k for k, v in _SN_CLASS.items()}
    for m in list(module.modules()):
        base = inverse.get(type(m))
        if base is None:
            continue
        m.weight.copy_(m.sn_weight())
        for name in ("sn_u", "sn_v", "sn_gain"):
            delattr(m, name)
        m.__class__ = base
        n += 1
    return n
