"""Training loops and the model registry."""
from .registry import build_model, register_model, registered_models

__all__ = ["build_model", "register_model", "registered_models"]
