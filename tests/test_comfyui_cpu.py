"""ComfyUI helpers without ComfyUI: the sigma grid and the re-noise rule."""
import torch


def test_dmad_sigmas():
    from dmad_b200.comfyui import dmad_sigmas

    s = dmad_sigmas(4, 12.0)
    assert s.shape == (5,) and s[0] == 1.0 and s[-1] == 0.0
    u = torch.tensor(0.75)
    assert torch.isclose(s[1], 12 * u / (1 + 11 * u))


def test_sample_dmad_renoise_rule():
    from dmad_b200.comfyui import dmad_sigmas, sample_dmad

    target = torch.full((2, 3), 0.5)
    seen = []

    def model(x, sig, seed=None):
        seen.append((x.clone(), sig.clone()))
        return target.clone()

    sig = dmad_sigmas(3, 1.0)
    x = sample_dmad(model, torch.randn(2, 3), sig, extra_args={"seed": 7})
    assert torch.equal(x, target) and len(seen) == 3
    g = torch.Generator().manual_seed(7)
    eps = torch.randn(2, 3, generator=g)
    s1 = float(sig[1])
    assert torch.allclose(seen[1][0], target * (1 - s1) + eps * s1)   # re-noised with fresh seeded noise
    x2 = sample_dmad(model, torch.randn(2, 3), sig, extra_args={"seed": 7})
    assert torch.equal(x2, x)
