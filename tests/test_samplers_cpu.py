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
