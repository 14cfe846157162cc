"""sm_100a kernels and their autograd wrappers.

Every op here has two implementations with identical math:

* CUDA tensors run the hand-written sm_100a kernels of ``dmad_b200._C``
  (built in-tree by ``setup.py build_ext --inplace``).  If the extension is
  missing on a GPU machine the op raises instead of silently falling back.
* CPU tensors run a plain PyTorch restatement of the same math.  It exists so
  the model, algorithm and distributed logic can be unit-tested without a GPU,
  and it is the fp32 oracle the kernel tests compare against.
"""
from __future__ import annotations

import importlib

import torch

_C = None
_C_ERR: Exception | None = None


def _load():
    global _C, _C_ERR
    if _C is None and _C_ERR is None:
        try:
            _C = importlib.import_module("dmad_b200._C")
        except Exception as e:  # pragma: no cover - depends on the build
            _C_ERR = e
    return _C


def native_available() -> bool:
    return _load() is not None


def ext():
    """The compiled extension; raises with the build hint when it is missing."""
    m = _load()
    if m is None:
        raise RuntimeError(
            "dmad_b200._C is not built (run `python setup.py build_ext --inplace`); "
            f"CUDA ops have no fallback. Import error: {_C_ERR!r}"
        )
    return m


def device_status(device: int | None = None, reset: bool = True) -> int:
    """Status word written by kernels whose bounded waits ran out (0 = ok)."""
    if device is None:
        device = torch.cuda.current_device()
    return int(ext().device_status(int(device), bool(reset)))


def check_device_status(device: int | None = None) -> None:
    code = device_status(device, reset=True)
    if code != 0:
        names = {1: "TMA load wait", 2: "MMA completion wait", 3: "softmax handoff wait",
                 4: "stage release wait", 5: "peer flag wait", 6: "bounds check"}
        raise RuntimeError(f"dmad kernel reported a bounded-wait failure: {names.get(code, code)} (code {code})")


from .attention import flash_attention, attention_reference, flash_attention_jvp, attention_jvp_reference  # noqa: E402
from .norm import ln_mod, gate_residual, qk_norm_rope, rope, rope_apply, rms_norm, layer_norm_affine  # noqa: E402
from .activation import gelu_tanh  # noqa: E402
from .temb import sinusoidal_embedding, small_linear  # noqa: E402

__all__ = [
    "native_available",
    "ext",
    "device_status",
    "check_device_status",
    "flash_attention",
    "flash_attention_jvp",
    "attention_jvp_reference",
    "attention_reference",
    "ln_mod",
    "gate_residual",
    "qk_norm_rope",
    "rope",
    "rope_apply",
    "rms_norm",
    "layer_norm_affine",
    "gelu_tanh",
    "sinusoidal_embedding",
    "small_linear",
]
