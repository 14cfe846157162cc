"""ComfyUI nodes: ``DMADSampler`` (re-noise multistep rule) and ``DMADSigmas`` (shifted grid).

Parity: comfyui/ComfyUI-DMAD/nodes.py:29-101.  The students are trained with the re-noise rule:
at every step the model's x0 prediction is re-noised with fresh noise at the next sigma,
``x_{i+1} = (1 - s_{i+1}) x0 + s_{i+1} eps`` (the last step returns x0), instead of following the
ODE.  The noise generator is seeded with the sampling seed, so a run is reproducible.

The two functions work without ComfyUI; the node classes are only defined when ComfyUI's
``comfy_api`` is importable (copy or symlink this directory into ``ComfyUI/custom_nodes``).
"""
from __future__ import annotations

import torch


def dmad_sigmas(steps: int, shift: float) -> torch.Tensor:
    """``steps + 1`` sigmas from 1 to 0: s(u) = shift u / (1 + (shift - 1) u) on a linear u grid."""
    u = torch.linspace(1.0, 0.0, steps + 1, dtype=torch.float32)
    return shift * u / (1.0 + (shift - 1.0) * u)


def _noise_like(x, gen):
    if getattr(x, "is_nested", False):  # ComfyUI's nested tensors (packed audio + video)
        import comfy.nested_tensor
        return comfy.nested_tensor.NestedTensor([torch.randn(t.shape, dtype=t.dtype, device=t.device, generator=gen)
                                                 for t in x.unbind()])
    return torch.randn(x.shape, dtype=x.dtype, device=x.device, generator=gen)


@torch.no_grad()
def sample_dmad(model, x, sigmas, extra_args=None, callback=None, disable=None):
    """Re-noise sampling with a denoiser ``model(x, sigma * ones(B), **extra_args) -> x0``."""
    extra_args = dict(extra_args or {})
    seed = extra_args.get("seed")
    gen = torch.Generator(device=x.device).manual_seed(int(seed)) if seed is not None else None
    ones = x.new_ones([x.shape[0]])
    steps = range(len(sigmas) - 1)
    if disable is False:
        from tqdm.auto import trange
        steps = trange(len(sigmas) - 1)
    for i in steps:
        x0 = model(x, sigmas[i] * ones, **extra_args)
        if callback is not None:
            callback({"x": x, "i": i, "sigma": sigmas[i], "sigma_hat": sigmas[i], "denoised": x0})
        nxt = float(sigmas[i + 1])
        x = x0 if nxt <= 0 else x0 * (1.0 - nxt) + _noise_like(x0, gen) * nxt
    return x


try:  # node definitions only under ComfyUI
    import comfy.samplers
    from comfy_api.latest import ComfyExtension, io

    class DMADSampler(io.ComfyNode):
        @classmethod
        def define_schema(cls):
            return io.Schema(node_id="DMADSampler", display_name="DMAD Sampler (re-noise)",
                             category="sampling/custom_sampling/samplers",
                             description="Denoise to x0, then re-noise with fresh noise at the next sigma (the rule the "
                                         "DMAD students were trained with). Use cfg 1.0 and the DMAD Sigmas node.",
                             inputs=[], outputs=[io.Sampler.Output()])

        @classmethod
        def execute(cls):
            return io.NodeOutput(comfy.samplers.KSAMPLER(sample_dmad))

    class DMADSigmas(io.ComfyNode):
        @classmethod
        def define_schema(cls):
            return io.Schema(node_id="DMADSigmas", display_name="DMAD Sigmas",
                             category="sampling/custom_sampling/schedulers",
                             description="Shifted linear grid from 1 to 0 (shift 12 for H3 video, audio shift 2).",
                             inputs=[io.Int.Input("steps", default=4, min=1, max=64),
                                     io.Float.Input("shift", default=12.0, min=0.01, max=100.0, step=0.01)],
                             outputs=[io.Sigmas.Output()])

        @classmethod
        def execute(cls, steps, shift):
            return io.NodeOutput(dmad_sigmas(steps, shift))

    class DMADExtension(ComfyExtension):
        async def get_node_list(self):
            return [DMADSampler, DMADSigmas]

    async def comfy_entrypoint():
        return DMADExtension()
except ImportError:  # not running inside ComfyUI
    pass
