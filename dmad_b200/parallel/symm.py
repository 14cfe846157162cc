"""Symmetric device buffers and a bounded-wait cross-GPU barrier.

A ``SymmBuffer`` is one allocation that every rank of the group maps: ``ptrs[r]`` is the
address of rank r's copy as seen from this GPU (NVLink peer mapping), and ``mc_ptr`` is
the NVSwitch multicast address of the whole group's copies when the fabric offers it
(``multimem`` loads there are summed in the switch, stores are replicated to every GPU).
With one process and no process group the buffer is an ordinary device tensor.

``PeerSync`` is the barrier the fused collective kernels put around their peer traffic.
Each rank writes an increasing epoch into a flag of every peer and waits (on the GPU, for at
most ``timeout_s``) until every peer's flag has reached it; a float payload can ride along
(used to exchange the partial gradient norms for clipping).  A wait that runs out sets the
device status word (``ops.check_device_status``) instead of hanging, and the optimiser kernels
that follow skip their update.

Plumbing only: the allocation and the exchange of the peer addresses use
``torch.distributed._symmetric_memory``; every load and store on the peer memory is issued by
the kernels in ``csrc/collectives.cu``.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from .dist import get_rank, get_world_size, is_distributed


def _group_name(group):
    g = group if group is not None else dist.group.WORLD
    return g.group_name


class SymmBuffer:
    def __init__(self, numel: int, dtype: torch.dtype, device, group=None, zero: bool = True):
        self.group = group
        self.world = get_world_size(group)
        self.rank = get_rank() if group is None else dist.get_rank(group)
        self.device = torch.device(device)
        self.handle = None
        if self.world == 1 or not is_distributed() or self.device.type != "cuda":
            self.tensor = torch.zeros(numel, dtype=dtype, device=self.device) if zero else \
                torch.empty(numel, dtype=dtype, device=self.device)
            self.ptrs = [self.tensor.data_ptr()] * self.world if self.device.type == "cuda" else []
            self.mc_ptr = 0
            return
        import torch.distributed._symmetric_memory as symm_mem

        self.tensor = symm_mem.empty(numel, dtype=dtype, device=self.device)
        if zero:
            self.tensor.zero_()
        self.handle = symm_mem.rendezvous(self.tensor, _group_name(group))
        base = list(self.handle.buffer_ptrs)
        off = self.tensor.data_ptr() - base[self.rank]
        self.ptrs = [int(b) + off for b in base]
        self.mc_ptr = 0
        try:  # 0 when the fabric / driver gives no multicast object
            mc = int(self.handle.multicast_ptr)
        except Exception:  # noqa: BLE001 - any failure means: no multicast
            mc = 0
        self.mc_ptr = mc + off if mc != 0 else 0


class PeerSync:
    """Bounded-wait barrier over a symmetric int32 buffer: flags[world] then float slots[world]."""

    def __init__(self, device, group=None, timeout_s: float = 120.0):
        self.world = get_world_size(group)
        self.rank = get_rank() if group is None else dist.get_rank(group)
        self.timeout_s = float(timeout_s)
        self.epoch = 0
        self.device = torch.device(device)
        self.buf = SymmBuffer(2 * max(self.world, 1) + 2, torch.int32, device, group)
        self.ptrs_dev = torch.tensor(self.buf.ptrs, dtype=torch.int64, device=self.device) \
            if self.device.type == "cuda" else None
        # every rank has zeroed its flags before any peer writes into them
        if is_distributed() and self.world > 1 and self.device.type == "cuda":
            from .dist import barrier
            torch.cuda.synchronize(self.device)
            barrier()

    @property
    def slots(self) -> torch.Tensor:
        """This rank's float slots (one per rank) filled by the payload of the last barrier."""
        return self.buf.tensor[self.world:2 * self.world].view(torch.float32)

    def __call__(self, payload: torch.Tensor | None = None):
        if self.world == 1 or self.device.type != "cuda":
            if payload is not None:
                self.slots[self.rank] = payload.reshape(-1)[0]
            return
        from ..ops import ext

        self.epoch += 1
        ext().symm_barrier(self.ptrs_dev, self.rank, self.epoch, payload, self.timeout_s)
