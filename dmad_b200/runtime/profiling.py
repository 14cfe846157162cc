"""Profiler and memory-snapshot contexts for training runs.

Parity: train/wan/imaginaire/utils/profiling.py:32-133 (``maybe_enable_profiling`` with a
wait / warmup / active schedule and per-rank trace files, ``maybe_enable_memory_snapshot``).
Enabled from the config section ``profiling``: ``enabled``, ``wait``, ``warmup``, ``active``,
``dir``, ``memory_snapshot``, ``ranks``.
"""
from __future__ import annotations

import contextlib
import os

import torch

from ..parallel.dist import get_rank


@contextlib.contextmanager
def maybe_profile(cfg: dict | None, start_iteration: int = 0):
    cfg = cfg or {}
    ranks = cfg.get("ranks", [0])
    if not cfg.get("enabled") or get_rank() not in ranks:
        yield None
        return
    from torch.profiler import ProfilerActivity, profile, schedule

    out_dir = cfg.get("dir", "profiles_run")
    os.makedirs(out_dir, exist_ok=True)

    def on_ready(prof):
        path = os.path.join(out_dir, f"trace_rank{get_rank()}_it{start_iteration + prof.step_num}.json")
        prof.export_chrome_trace(path)
        with open(os.path.join(out_dir, f"table_rank{get_rank()}.txt"), "w") as f:
            f.write(prof.key_averages().table(sort_by="cuda_time_total" if torch.cuda.is_available()
                                              else "cpu_time_total", row_limit=60))

    acts = [ProfilerActivity.CPU] + ([ProfilerActivity.CUDA] if torch.cuda.is_available() else [])
    with profile(activities=acts, record_shapes=bool(cfg.get("record_shapes", False)),
                 schedule=schedule(wait=int(cfg.get("wait", 1)), warmup=int(cfg.get("warmup", 1)),
                                   active=int(cfg.get("active", 2)), repeat=1),
                 on_trace_ready=on_ready) as prof:
        yield prof


@contextlib.contextmanager
def maybe_memory_snapshot(cfg: dict | None):
    cfg = cfg or {}
    if not cfg.get("memory_snapshot") or not torch.cuda.is_available() or get_rank() not in cfg.get("ranks", [0]):
        yield None
        return
    out_dir = cfg.get("dir", "profiles_run")
    os.makedirs(out_dir, exist_ok=True)
    torch.cuda.memory._record_memory_history(max_entries=int(cfg.get("max_entries", 100000)))
    try:
        yield True
    finally:
        torch.cuda.memory._dump_snapshot(os.path.join(out_dir, f"memory_rank{get_rank()}.pickle"))
        torch.cuda.memory._record_memory_history(enabled=None)
