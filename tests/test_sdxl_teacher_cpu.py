"""SDXL teacher-latent generation (parity: train/image/main/sdxl/generate_teacher_latents.py): the
trailing Euler schedule, an exact-denoiser check of the sampler, and resumable chunked generation merged
into the latent/prompt LMDB layout (a dictionary-backed stand-in for the lmdb package)."""
import numpy as np
import torch

from test_lmdb_cpu import _Env


def test_trailing_schedule():
    from dmad_b200.models.sdxl import ddpm_alphas_cumprod
    from dmad_b200.tools.sdxl_teacher_latents import euler_trailing_schedule

    ts, sig = euler_trailing_schedule(50)
    assert ts[0] == 999 and ts[1] == 979 and ts[-1] == 19 and len(sig) == 51 and sig[-1] == 0
    ac = ddpm_alphas_cumprod()
    assert abs(float(sig[0]) - float(((1 - ac[999]) / ac[999]) ** 0.5)) < 1e-4
    assert bool((sig[:-1] > sig[1:]).all())


def test_euler_with_an_exact_denoiser_reaches_the_data_point():
    """Data = a point mass at 0: the exact epsilon at (x, sigma) is x / sigma, and the Euler chain lands
    on 0 at sigma = 0 whatever the guidance."""
    from dmad_b200.tools.sdxl_teacher_latents import euler_trailing_schedule, sample_latents

    ts, sig = euler_trailing_schedule(10)

    class Exact(torch.nn.Module):
        def __init__(self):
            super().__init__()
            self.w = torch.nn.Parameter(torch.zeros(1))

        def forward(self, x_in, t, ctx, ids, pooled):
            s = sig[(ts - t[0]).abs().argmin()]
            return x_in * (s ** 2 + 1) ** 0.5 / s  # x / sigma from the scaled input

    x = sample_latents(Exact(), torch.randn(2, 77, 16), torch.randn(2, 8), steps=10, guidance=8.0, resolution=64,
                       generator=torch.Generator().manual_seed(0))
    assert x.shape == (2, 4, 8, 8) and float(x.abs().max()) < 1e-4


def test_chunked_generation_and_merge():
    from dmad_b200.data.lmdb_arrays import LMDBLatentPromptDataset, write_rows, write_shapes
    from dmad_b200.models.sdxl import SDXLUNet
    from dmad_b200.tools.sdxl_teacher_latents import generate, load_prompts, merge

    real = _Env()
    lat = np.zeros((5, 4, 8, 8), np.float16)
    write_rows(real, {"latents": lat, "prompts": [f"caption {i}" for i in range(5)]})
    write_shapes(real, {"latents": lat}, 5)
    prompts = load_prompts(real)
    torch.manual_seed(0)
    unet = SDXLUNet(channels=(32, 64), depths=(0, 1), ctx_dim=16, pooled_dim=8, addition_time_embed_dim=8,
                    layers_per_block=1).eval()
    enc = lambda ps: (torch.randn(len(ps), 77, 16), torch.randn(len(ps), 8))  # noqa: E731
    import tempfile
    with tempfile.TemporaryDirectory() as d:
        for shard in range(2):
            w = generate(unet, enc, prompts, d, shard, 2, batch=2, chunk=2, steps=2, resolution=64)
            assert len(w) == (2 if shard == 0 else 1)
        assert generate(unet, enc, prompts, d, 0, 2, batch=2, chunk=2, steps=2, resolution=64) == []  # resumable
        out = _Env()
        assert merge(d, out) == 5
    ds = LMDBLatentPromptDataset(out)
    assert len(ds) == 5 and [ds[i]["prompt"] for i in range(5)] == prompts
    assert ds[3]["images"].shape == (4, 8, 8) and torch.isfinite(ds[3]["images"]).all()
