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


class EveryNDrawSample(Callback):
    """Every ``every`` iterations, few-step samples of the current batch's prompts (1, 2 and
    ``num_steps`` steps, live or EMA student) saved as latents to ``<out_dir>/samples``.

    Parity: train/wan/rcm/callbacks/every_n_draw_distill.py:102-247 (1-, 2- and N-step samples of the
    training batch, ``is_ema`` tag, only the first ``n_sample_to_save`` data-parallel ranks write).  Every
    rank samples, so context-parallel groups stay in step; the latents are written instead of decoded
    video (decode them with ``cli.wan_sample``'s VAE path)."""

    def __init__(self, out_dir: str, every: int, num_steps: int = 4, is_ema: bool = False, n_ranks_to_save: int = 1,
                 run_at_start: bool = False, seed: int = 0):
        self.out_dir, self.every, self.num_steps = out_dir, int(every), int(num_steps)
        self.is_ema, self.n_ranks, self.run_at_start, self.seed = is_ema, int(n_ranks_to_save), run_at_start, seed
        self.written: list = []

    def on_train_start(self, trainer, iteration):
        self._start = iteration

    def on_step_end(self, trainer, iteration, out):
        if self.every <= 0 or iteration % self.every or (iteration == self._start and not self.run_at_start):
            return None
        gen = getattr(trainer.model, "generate", None)
        batch = getattr(trainer, "last_batch", None)
        if gen is None or not isinstance(batch, dict) or "latents" not in batch or "context" not in batch:
            return None
        import os

        lat, ctx = batch["latents"], batch["context"]
        device = lat.device
        g = torch.Generator(device=device).manual_seed(self.seed)
        samples = {}
        with torch.no_grad():
            for n in sorted({1, 2, self.num_steps}):
                g.manual_seed(self.seed)
                samples[f"steps_{n}"] = gen(ctx, tuple(lat.shape), num_steps=n, generator=g,
                                            use_ema=self.is_ema).float().cpu()
        rank = getattr(trainer, "rank", 0)
        if rank < self.n_ranks:
            tag = "ema" if self.is_ema else "reg"
            os.makedirs(os.path.join(self.out_dir, "samples"), exist_ok=True)
            path = os.path.join(self.out_dir, "samples", f"iter_{iteration:09d}_{tag}_rank{rank:03d}.pt")
            torch.save({"iteration": iteration, "tag": tag, **samples}, path)
            self.written.append(path)
        return None
