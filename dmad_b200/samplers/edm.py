"""EDM teacher sampler and Frechet distance (image stack).

* ``edm_sigmas`` / ``edm_heun_sampler`` -- the stochastic Heun sampler of Karras et al., "Elucidating the
  Design Space of Diffusion-Based Generative Models" (NeurIPS 2022), Algorithm 2: Karras sigma grid
  with exponent rho, churn gamma = min(S_churn / N, sqrt(2) - 1) inside [S_min, S_max], noise
  inflation S_noise, Euler step with a second-order correction except at the last step.  The
  reference's teacher samples use 256 steps, S_churn 40, S_min 0.05, S_max 50, S_noise 1.003, seed
  per sample (train/image/main/edm/generate_teacher_samples.py:59-90).
* ``frechet_distance`` / ``feature_stats`` -- FID between Gaussian fits of two feature sets,
  ||mu1 - mu2||^2 + Tr(S1 + S2 - 2 (S1 S2)^(1/2)) (Heusel et al. 2017), as the reference's FID
  evaluation computes it on Inception features (:93-99, test_folder_edm.py).  The feature extractor
  is the caller's (no Inception weights ship with this repository).
"""
from __future__ import annotations

import numpy as np
import torch


def edm_sigmas(steps: int, sigma_min: float = 0.002, sigma_max: float = 80.0, rho: float = 7.0, device=None):
    i = torch.arange(steps, dtype=torch.float64, device=device)
    s = (sigma_max ** (1 / rho) + i / max(steps - 1, 1) * (sigma_min ** (1 / rho) - sigma_max ** (1 / rho))) ** rho
    return torch.cat([s, torch.zeros(1, dtype=torch.float64, device=device)])


@torch.no_grad()
def edm_heun_sampler(denoise, latents, class_labels=None, steps: int = 256, sigma_min=0.002, sigma_max=80.0,
                     rho=7.0, S_churn=40.0, S_min=0.05, S_max=50.0, S_noise=1.003, randn_like=torch.randn_like):
    """``denoise(x, sigma, labels) -> x0``; ``latents`` ~ N(0, I).  Returns the fp64 sample."""
    t = edm_sigmas(steps, sigma_min, sigma_max, rho, latents.device)
    x = latents.double() * t[0]
    for i in range(steps):
        tc, tn = t[i], t[i + 1]
        gamma = min(S_churn / steps, np.sqrt(2) - 1) if S_min <= float(tc) <= S_max else 0.0
        th = tc + gamma * tc
        xh = x + (th ** 2 - tc ** 2).sqrt() * S_noise * randn_like(x)
        d = (xh - denoise(xh.float(), th.float(), class_labels).double()) / th
        xn = xh + (tn - th) * d
        if i < steps - 1:
            d2 = (xn - denoise(xn.float(), tn.float(), class_labels).double()) / tn
            xn = xh + (tn - th) * (0.5 * d + 0.5 * d2)
        x = xn
    return x


def feature_stats(features) -> tuple[np.ndarray, np.ndarray]:
    f = np.asarray(features, dtype=np.float64)
    return f.mean(0), np.cov(f, rowvar=False)


def frechet_distance(mu1, sigma1, mu2, sigma2) -> float:
    from scipy import linalg

    diff = np.asarray(mu1) - np.asarray(mu2)
    covmean = linalg.sqrtm(np.asarray(sigma1) @ np.asarray(sigma2))
    if not np.isfinite(covmean).all():
        eps = np.eye(len(mu1)) * 1e-6
        covmean = linalg.sqrtm((sigma1 + eps) @ (sigma2 + eps))
    return float(diff @ diff + np.trace(sigma1) + np.trace(sigma2) - 2 * np.trace(np.real(covmean)))
