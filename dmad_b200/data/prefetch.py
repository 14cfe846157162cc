"""Host -> device batch prefetch on a side stream.

The next batch is copied from pinned host memory with ``non_blocking`` copies on a dedicated
CUDA stream while the current step runs; the compute stream waits on an event before using it
(the reference hands pinned batches from its DataLoader to ``misc.to(..., device)`` on the compute
stream, train/wan/rcm/trainers/trainer_distillation.py:185-196).
"""
from __future__ import annotations

import torch


def _pin(x):
    if torch.is_tensor(x):
        return x.pin_memory() if not x.is_pinned() else x
    if isinstance(x, dict):
        return {k: _pin(v) for k, v in x.items()}
    return x


def _to(x, device, non_blocking=True):
    if torch.is_tensor(x):
        return x.to(device, non_blocking=non_blocking)
    if isinstance(x, dict):
        return {k: _to(v, device, non_blocking) for k, v in x.items()}
    return x


class DevicePrefetcher:
    def __init__(self, iterable, device, rename: dict | None = None):
        self.it = iter(iterable)
        self.device = torch.device(device)
        self.rename = rename or {}
        self.cuda = self.device.type == "cuda"
        self.stream = torch.cuda.Stream(device=self.device) if self.cuda else None
        self._next = None
        self._event = None
        self._preload()

    def _preload(self):
        try:
            host = next(self.it)
        except StopIteration:
            self._next = None
            return
        host = {self.rename.get(k, k): v for k, v in host.items()}
        if not self.cuda:
            self._next = host
            return
        host = _pin(host)
        with torch.cuda.stream(self.stream):
            self._next = _to(host, self.device)
            self._event = torch.cuda.Event()
            self._event.record(self.stream)

    def __iter__(self):
        return self

    def __next__(self):
        if self._next is None:
            raise StopIteration
        if self.cuda:
            torch.cuda.current_stream(self.device).wait_event(self._event)
            for v in self._next.values():
                if torch.is_tensor(v):
                    v.record_stream(torch.cuda.current_stream(self.device))
        batch = self._next
        self._preload()
        return batch
