"""Smaller runtime pieces on CPU: device prefetcher, trainer callbacks (NVML through a fake), the
profiler context, the experiment presets through the config loader, the model registry, and the H3
inference CLI on a tiny random model."""
import json
import os

import pytest
import torch


def test_prefetcher_renames_and_yields_in_order():
    from dmad_b200.data.prefetch import DevicePrefetcher

    data = [{"a": torch.full((2,), float(i)), "b": i} for i in range(3)]
    out = list(DevicePrefetcher(data, "cpu", rename={"a": "x"}))
    assert [int(o["x"][0]) for o in out] == [0, 1, 2] and [o["b"] for o in out] == [0, 1, 2]


def test_callbacks():
    from dmad_b200.runtime.callbacks import DataLoadingSpeed, DeviceMonitor, ForceFiniteLoss, IterSpeed, ManualGC

    class Mem:
        used = 3 * 2 ** 30

    class Util:
        gpu = 55

    class FakeNVML:
        def nvmlInit(self):
            pass

        def nvmlDeviceGetHandleByIndex(self, i):
            return ("gpu", i)

        def nvmlDeviceGetMemoryInfo(self, h):
            return Mem()

        def nvmlDeviceGetUtilizationRates(self, h):
            return Util()

        def nvmlDeviceGetPowerUsage(self, h):
            return 612000

    it = IterSpeed(every=2)
    it.on_train_start(None, 0)
    assert it.on_step_end(None, 1, {}) is None and "speed/iter_s" in it.on_step_end(None, 2, {})
    dl = DataLoadingSpeed()
    dl.on_before_dataloading(None, 0)
    dl.on_after_dataloading(None, 0)
    assert dl.on_step_end(None, 0, {})["speed/data_s"] >= 0
    dm = DeviceMonitor(every=1, nvml=FakeNVML()).on_step_end(None, 1, {})
    assert dm["device/power_w"] == 612.0 and dm["device/util_pct"] == 55.0 and dm["device/mem_used_gib"] == 3.0
    assert ForceFiniteLoss().on_step_end(None, 0, {"l": torch.tensor(float("nan")), "m": torch.tensor(1.0)}) == \
        {"health/nonfinite_outputs": 1.0}
    gcb = ManualGC(every=1)
    gcb.on_train_start(None, 0)
    gcb.on_step_end(None, 1, {})
    gcb.on_train_end(None, 1)
    import gc
    assert gc.isenabled()


def test_profiler_context_writes_table(tmp_path):
    from dmad_b200.runtime.profiling import maybe_profile

    with maybe_profile({"enabled": True, "wait": 0, "warmup": 0, "active": 1, "dir": str(tmp_path)}) as prof:
        for _ in range(2):
            torch.randn(64, 64) @ torch.randn(64, 64)
            prof.step()
    assert (tmp_path / "table_rank0.txt").exists()
    with maybe_profile(None) as prof:
        assert prof is None


def test_presets_and_registry():
    import dmad_b200.cli.presets  # noqa: F401  (registers the experiments)
    from dmad_b200.runtime.config import experiments, load_config
    from dmad_b200.train.registry import registered_models

    assert {"dmad_wan2pt1_1pt3b", "dmad_wan2pt1_14b_cp8", "rcm_wan2pt1_1pt3b", "dmad_wan2pt1_1pt3b_debug"} <= set(experiments())
    assert load_config(None, ["experiment=dmad_wan2pt1_1pt3b_debug"])["training"]["max_iters"] == 25
    cfg = load_config(None, ["experiment=dmad_wan2pt1_14b_cp8", "training.max_iters=3"])
    assert cfg["parallel"]["cp"] == 8 and cfg["training"]["max_iters"] == 3
    assert cfg["model"]["distill"]["checkpoint_student_policy"] == "mm_only"
    assert {"wan_dmad", "h3_dmad", "edm_dmad", "sdxl_dmad"} <= set(registered_models())


def test_h3_inference_cli_tiny(tmp_path):
    from dmad_b200.cli.h3_inference import main

    (tmp_path / "p.txt").write_text("a fox\n", encoding="utf-8")
    main(["--random-init", "--config", "tiny", "--prompt-file", str(tmp_path / "p.txt"), "--output-dir",
          str(tmp_path / "out"), "--steps", "1", "--height", "64", "--width", "64", "--num-frames", "22",
          "--text-tokens", "4"])
    files = os.listdir(tmp_path / "out")
    assert files, "no output written"
