"""Trainer callbacks (hooks around every iteration).

Parity: the Wan callback set (train/wan/rcm/callbacks/*, configured in
train/wan/rcm/configs/defaults/callbacks.py:17-73): ``IterSpeed``, ``DeviceMonitor`` (power and
memory through NVML, read only), ``GradClip``'s force-finite + norm logging, ``HeartBeat``,
``ManualGarbageCollection``, ``DetailedDataLoadingSpeedMonitor`` and ``DMADScalars`` (the last is
``runtime.logging.MetricsWriter``).  ``LowPrecisionCallback`` has no counterpart: the fused
optimiser kernels write the bf16 weights from the fp32 master in the same pass.
"""
from __future__ import annotations

import gc
import time

import torch


class Callback:
    def on_train_start(self, trainer, iteration: int):
        pass

    def on_before_dataloading(self, trainer, iteration: int):
        pass

    def on_after_dataloading(self, trainer, iteration: int):
        pass

    def on_step_end(self, trainer, iteration: int, out: dict) -> dict | None:
        """May return extra scalars for the metrics window."""
        return None

    def on_train_end(self, trainer, iteration: int):
        pass


class IterSpeed(Callback):
    """Wall time per iteration (host clock, synchronised every ``every`` iterations)."""

    def __init__(self, every: int = 10):
        self.every = every
        self._t = None
        self._it = 0

    def on_train_start(self, trainer, iteration):
        self._t, self._it = time.perf_counter(), iteration

    def on_step_end(self, trainer, iteration, out):
        if iteration % self.every:
            return None
        if torch.cuda.is_available():
            torch.cuda.synchronize()
        now = time.perf_counter()
        dt = (now - self._t) / max(1, iteration - self._it)
        self._t, self._it = now, iteration
        return {"speed/iter_s": dt}


class DataLoadingSpeed(Callback):
    def __init__(self):
        self._t0 = 0.0
        self.last = 0.0

    def on_before_dataloading(self, trainer, iteration):
        self._t0 = time.perf_counter()

    def on_after_dataloading(self, trainer, iteration):
        self.last = time.perf_counter() - self._t0

    def on_step_end(self, trainer, iteration, out):
        return {"speed/data_s": self.last}


class DeviceMonitor(Callback):
    """GPU power, utilisation and memory through NVML (reads only; changes no GPU setting)."""

    def __init__(self, every: int = 50, nvml=None):
        self.every = every
        self._nvml = nvml
        self._h = None

    def _handle(self):
        if self._h is None:
            if self._nvml is None:
                import pynvml as nvml  # nvidia-ml-py
                self._nvml = nvml
            self._nvml.nvmlInit()
            idx = torch.cuda.current_device() if torch.cuda.is_available() else 0
            self._h = self._nvml.nvmlDeviceGetHandleByIndex(idx)
        return self._h

    def on_step_end(self, trainer, iteration, out):
        if iteration % self.every:
            return None
        try:
            h = self._handle()
            nv = self._nvml
            mem = nv.nvmlDeviceGetMemoryInfo(h)
            util = nv.nvmlDeviceGetUtilizationRates(h)
            return {"device/power_w": nv.nvmlDeviceGetPowerUsage(h) / 1000.0, "device/util_pct": float(util.gpu),
                    "device/mem_used_gib": mem.used / 2 ** 30,
                    "device/max_alloc_gib": (torch.cuda.max_memory_allocated() / 2 ** 30
                                             if torch.cuda.is_available() else 0.0)}
        except Exception:  # noqa: BLE001 - no NVML on this host
            return None


class ManualGC(Callback):
    """Python garbage collection at fixed intervals instead of at random points of a step."""

    def __init__(self, every: int = 50):
        self.every = every

    def on_train_start(self, trainer, iteration):
        gc.disable()

    def on_step_end(self, trainer, iteration, out):
        if iteration % self.every == 0:
            gc.collect(1)
        return None

    def on_train_end(self, trainer, iteration):
        gc.enable()


class HeartBeatCallback(Callback):
    """Publishes this rank's heartbeat and checks the peers' between iterations."""

    def __init__(self, heartbeat, max_age_s: float):
        self.hb = heartbeat
        self.max_age = max_age_s

    def on_train_start(self, trainer, iteration):
        self.hb.start()

    def on_before_dataloading(self, trainer, iteration):
        self.hb.check(self.max_age)

    def on_train_end(self, trainer, iteration):
        self.hb.stop()


class ForceFiniteLoss(Callback):
    """Counts non-finite losses in a step's outputs (the reference's GradClip force-finite log)."""

    def on_step_end(self, trainer, iteration, out):
        bad = 0
        for k, v in out.items():
            if torch.is_tensor(v) and v.is_floating_point() and not torch.isfinite(v).all():
                bad += 1
        return {"health/nonfinite_outputs": float(bad)}
