"""Noise-time parameterisations and samplers.

Parity: train/wan/rcm/utils/timestep_utils.py:7-120 (RF / sigma / TrigFlow conversions,
LogNormal and UniformShift samplers with CDF / inverse CDF) and
train/wan/rcm/utils/denoiser_scaling.py:19-30 (TrigFlow preconditioning of a
rectified-flow network).
"""
from __future__ import annotations

import math

import torch


def shift_rf_time(u, shift: float):
    if shift <= 0:
        return u
    return shift * u / (1 + (shift - 1) * u)


def inverse_shift_rf_time(rf_t, shift: float):
    if shift <= 0:
        return rf_t
    return rf_t / (shift - (shift - 1.0) * rf_t)


def sigma_to_rf_time(sigma):
    return sigma / (sigma + 1)


def rf_to_sigma(rf_t):
    eps = torch.finfo(rf_t.dtype).eps
    rf_t = rf_t.clamp(min=0.0, max=1.0 - eps)
    return rf_t / (1 - rf_t)


def rf_to_trig_time(rf_t):
    return torch.arctan(rf_to_sigma(rf_t))


def trig_to_rf_time(trig_t):
    return sigma_to_rf_time(torch.tan(trig_t))


def _clamp01(x):
    eps = torch.finfo(x.dtype).eps
    return x.clamp(min=eps, max=1.0 - eps)


class LogNormal:
    """log(sigma) ~ N(p_mean, p_std); returns RF time sigma / (1 + sigma)."""

    def __init__(self, p_mean: float = 0.0, p_std: float = 1.0):
        self.p_mean, self.p_std = p_mean, p_std

    def __call__(self, shape, device="cpu", dtype=torch.float64, generator=None):
        z = torch.randn(shape, device=device, generator=generator).to(dtype)
        return sigma_to_rf_time(torch.exp(z * self.p_std + self.p_mean))

    def cdf_rf(self, rf_t):
        rf_t = _clamp01(rf_t)
        z = (torch.log(rf_t) - torch.log1p(-rf_t) - self.p_mean) / self.p_std
        return 0.5 * (1.0 + torch.erf(z / math.sqrt(2.0)))

    def icdf_rf(self, u):
        z = self.p_mean + self.p_std * math.sqrt(2.0) * torch.erfinv(2.0 * _clamp01(u) - 1.0)
        return torch.sigmoid(z)


class UniformShift:
    """u ~ U[0, 1) pushed through the flow shift s*u / (1 + (s-1) u)."""

    def __init__(self, shift: float = 0.0):
        self.shift = shift

    def __call__(self, shape, device="cpu", dtype=torch.float64, generator=None):
        u = torch.rand(shape, device=device, generator=generator).to(dtype)
        return shift_rf_time(u, self.shift)

    def cdf_rf(self, rf_t):
        return inverse_shift_rf_time(rf_t.clamp(0.0, 1.0), self.shift)

    def icdf_rf(self, u):
        return shift_rf_time(u.clamp(0.0, 1.0), self.shift)


class TrigFlowScaling:
    """(c_skip, c_out, c_in, c_noise) for a rectified-flow network driven with TrigFlow time t:
    x0 = c_skip x_t + c_out F(c_in x_t, c_noise); c_noise = sin/(cos+sin) * t_scale (the RF time x1000)."""

    def __init__(self, sigma_data: float = 1.0, t_scaling_factor: float = 1000.0):
        assert abs(sigma_data - 1.0) < 1e-6
        self.t_scaling_factor = t_scaling_factor

    def __call__(self, trig_t):
        t = trig_t.to(torch.float64)
        c, s = torch.cos(t), torch.sin(t)
        d = c + s
        return 1 / d, -s / d, 1 / d, (s / d) * self.t_scaling_factor
