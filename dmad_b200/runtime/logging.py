"""Rank-aware logging and JSONL metrics.

Parity: the H3 loguru setup with a rank filter and a file sink (train/h3/lightx2v_train/runtime/
logger.py:14-57), the optional experiment monitor (runtime/monitor.py:9-71; SwanLab / wandb there,
a JSONL file here) and the Wan ``DMADScalars`` callback that averages ``dmad*`` outputs over the
logging window and the ranks (train/wan/rcm/callbacks/*).
"""
from __future__ import annotations

import json
import logging
import os
import sys
import time

import torch

from ..parallel.dist import get_rank, get_world_size, is_distributed

_FMT = "%(asctime)s [rank%(rank)d] %(levelname)s %(name)s: %(message)s"


class _RankFilter(logging.Filter):
    def __init__(self, all_ranks: bool):
        super().__init__()
        self.all_ranks = all_ranks

    def filter(self, record):
        record.rank = get_rank()
        return self.all_ranks or record.rank == 0 or record.levelno >= logging.WARNING


def get_logger(name: str = "dmad_b200", log_file: str | None = None, all_ranks: bool = False,
               level: int = logging.INFO) -> logging.Logger:
    """Console logger (rank 0 only below WARNING unless ``all_ranks``) plus an optional per-rank file."""
    lg = logging.getLogger(name)
    if not getattr(lg, "_dmad_configured", False):
        lg.setLevel(level)
        lg.propagate = False
        h = logging.StreamHandler(sys.stderr)
        h.setFormatter(logging.Formatter(_FMT))
        h.addFilter(_RankFilter(all_ranks))
        lg.addHandler(h)
        lg._dmad_configured = True
    if log_file:
        path = log_file.replace("{rank}", str(get_rank()))
        if not any(isinstance(x, logging.FileHandler) and x.baseFilename == os.path.abspath(path) for x in lg.handlers):
            os.makedirs(os.path.dirname(os.path.abspath(path)), exist_ok=True)
            fh = logging.FileHandler(path)
            fh.setFormatter(logging.Formatter(_FMT))
            fh.addFilter(_RankFilter(True))
            lg.addHandler(fh)
    return lg


class MetricsWriter:
    """Averages scalars over a logging window and over ranks; rank 0 appends JSON lines."""

    def __init__(self, path: str | None, every: int = 10, prefixes: tuple = ()):
        self.path = path
        self.every = max(1, int(every))
        self.prefixes = tuple(prefixes)
        self._sum: dict[str, float] = {}
        self._cnt: dict[str, int] = {}
        self._t0 = time.time()
        if path and get_rank() == 0:
            os.makedirs(os.path.dirname(os.path.abspath(path)), exist_ok=True)

    def add(self, metrics: dict):
        for k, v in metrics.items():
            if self.prefixes and not k.startswith(self.prefixes):
                continue
            if torch.is_tensor(v):
                if v.numel() != 1:
                    continue
                v = float(v.detach().float().item())
            elif not isinstance(v, (int, float)):
                continue
            self._sum[k] = self._sum.get(k, 0.0) + float(v)
            self._cnt[k] = self._cnt.get(k, 0) + 1

    def should_flush(self, iteration: int) -> bool:
        return iteration % self.every == 0

    def flush(self, iteration: int, extra: dict | None = None) -> dict:
        """Collective when distributed (one all_reduce of the window means)."""
        keys = sorted(self._sum)
        means = [self._sum[k] / max(1, self._cnt[k]) for k in keys]
        if is_distributed() and get_world_size() > 1 and keys:
            import torch.distributed as dist

            dev = torch.device("cuda", torch.cuda.current_device()) if torch.cuda.is_available() and \
                dist.get_backend() == "nccl" else torch.device("cpu")
            t = torch.tensor(means, dtype=torch.float64, device=dev)
            dist.all_reduce(t)
            means = (t / get_world_size()).tolist()
        rec = {"iteration": iteration, "time": time.time(), "window_s": time.time() - self._t0}
        rec.update(dict(zip(keys, means)))
        if extra:
            rec.update(extra)
        self._sum.clear()
        self._cnt.clear()
        self._t0 = time.time()
        if self.path and get_rank() == 0:
            with open(self.path, "a") as f:
                f.write(json.dumps(rec) + "\n")
        return rec
