"""Flow samplers on Gaussian data, where the probability-flow ODE has a closed form: data
N(mu, s^2) reaches x(0) = mu + s * x(1).  Both samplers converge; UniPC (order 2, bh2) is far more
accurate than Euler at the same step count, and classifier-free guidance mixes velocities."""
import torch


def _velocity(mu, s):
    def v(x, t):
        sig = float(t) / 1000.0
        a = 1.0 - sig
        var = a * a * s * s + sig * sig
        x0 = mu + a * s * s / var * (x - a * mu)   # E[x0 | x_sigma]
        eps = (x - a * x0) / max(sig, 1e-12)
        return eps - x0
    return v


def test_flow_samplers_converge_to_exact_map():
    from dmad_b200.samplers import sample_flow

    torch.manual_seed(0)
    mu, s = 1.5, 0.3
    noise = torch.randn(4096, dtype=torch.float64)
    exact = mu + s * noise
    errs = {}
    for name in ("euler", "unipc"):
        for n in (16, 32, 64):
            x = sample_flow(_velocity(mu, s), noise.clone(), num_steps=n, shift=3.0, sampler=name)
            errs[(name, n)] = (x - exact).abs().max().item()
    # Euler is first order: halving the step halves the error
    assert 0.4 < errs[("euler", 64)] / errs[("euler", 32)] < 0.6, errs
    # UniPC (order 2 with corrector) converges faster and is more accurate at every count
    assert errs[("unipc", 64)] / errs[("unipc", 32)] < 0.25, errs
    for n in (16, 32, 64):
        assert errs[("unipc", n)] < errs[("euler", n)], errs
    assert errs[("unipc", 64)] < 1e-2, errs


def test_guidance_mixes_velocities():
    from dmad_b200.samplers import sample_flow

    noise = torch.zeros(3, dtype=torch.float64)
    vc = lambda x, t: torch.full_like(x, -2.0)  # noqa: E731
    vu = lambda x, t: torch.full_like(x, -1.0)  # noqa: E731
    x = sample_flow(vc, noise, num_steps=10, shift=1.0, sampler="euler", guidance=3.0, uncond_velocity_fn=vu)
    # v = -1 + 3 * (-2 + 1) = -4 integrated over sigma 1 -> 0 gives +4
    assert torch.allclose(x, torch.full_like(x, 4.0))


def test_edm_heun_gaussian_data():
    """With the exact denoiser of N(mu, s^2) data the deterministic EDM sampler (no churn) follows the
    probability-flow map, which keeps the standardised coordinate (x - mu) / sqrt(s^2 + sigma^2): a
    start x = sigma_max z ends at mu + s (sigma_max z - mu) / sqrt(s^2 + sigma_max^2).  With churn the
    samples have the data marginal; FID of identical Gaussians is ~0."""
    import numpy as np
    from dmad_b200.samplers.edm import edm_heun_sampler, feature_stats, frechet_distance

    mu, s = 0.7, 0.4

    def denoise(x, sigma, labels):
        sig = float(sigma)
        return mu + s * s / (s * s + sig * sig) * (x - mu)

    torch.manual_seed(0)
    z = torch.randn(20000, dtype=torch.float64)
    exact = mu + s * (80.0 * z - mu) / (80.0 ** 2 + s * s) ** 0.5
    e40 = (edm_heun_sampler(denoise, z, steps=40, S_churn=0.0) - exact).abs().max().item()
    e80 = (edm_heun_sampler(denoise, z, steps=80, S_churn=0.0) - exact).abs().max().item()
    assert e80 / e40 < 0.3 and e80 < 5e-3  # second order (Heun)
    x2 = edm_heun_sampler(denoise, z, steps=80, S_churn=40.0)   # stochastic: the data marginal
    assert abs(x2.mean().item() - mu) < 0.02 and abs(x2.std().item() - s) < 0.03
    f = np.random.default_rng(0).normal(size=(5000, 4))
    m, c = feature_stats(f)
    assert frechet_distance(m, c, m, c) < 1e-6
    assert abs(frechet_distance(m, c, m + 1.0, c) - 4.0) < 1e-6
