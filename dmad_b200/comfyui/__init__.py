"""ComfyUI integration: the DMAD re-noise sampler and the students' sigma grid as ComfyUI nodes."""
from .nodes import dmad_sigmas, sample_dmad

__all__ = ["dmad_sigmas", "sample_dmad"]
