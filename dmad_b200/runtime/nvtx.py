"""NVTX ranges around the fused kernels and collectives (visible in Nsight timelines).

Enabled with ``DMAD_NVTX=1`` (a range push / pop costs a few microseconds of host time, so it is
off by default).  Parity: the NVTX range context of train/wan/imaginaire/utils/misc.py:497-525.
"""
from __future__ import annotations

import contextlib
import os

import torch

ENABLED = os.environ.get("DMAD_NVTX", "0") not in ("", "0")


@contextlib.contextmanager
def nvtx_range(name: str):
    if ENABLED and torch.cuda.is_available():
        torch.cuda.nvtx.range_push(name)
        try:
            yield
        finally:
            torch.cuda.nvtx.range_pop()
    else:
        yield
