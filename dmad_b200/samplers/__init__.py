"""Teacher / baseline samplers for flow-matching models."""
from .flow import FlowEulerSampler, FlowUniPCSampler, sample_flow, shifted_sigmas

__all__ = ["FlowEulerSampler", "FlowUniPCSampler", "sample_flow", "shifted_sigmas"]
