"""Low-VRAM inference: stream transformer blocks host -> device one layer ahead of compute.

Parity with dmad_h3/lowmem.py (Streamer :176-331, AdaLNTables :400-413, TextLookup :464-475,
LowMemTransformer :478-574):
* every block's weights (minus its adaLN projection) live in one flat pinned host buffer;
* two rotating GPU slots; a worker thread issues ``cudaMemcpyAsync`` (``copy_(non_blocking=True)``) of
  block i+2 on a side stream once the compute stream has recorded that the slot's previous occupant is
  done; a forward pre-hook makes the compute stream wait on the copy and binds the parameters as views
  into the slot, the post-hook records ``compute_done`` and unbinds;
* the adaLN projections (the bulk of the parameters) depend only on the sampling step, so their outputs
  are tabulated per step up front and the projections are never streamed;
* the token refiner sees only the text, so its output is computed once per prompt;
* optional int8 per-output-row codec, dequantised to bf16 on the GPU right before use (changes the
  samples; off by default).
The kernels and their order are those of the resident model, so without the codec the output is
bit-identical to the resident run.
"""
from __future__ import annotations

import queue
import threading

import torch
import torch.nn as nn

_ALIGN = 256


def _aligned(n):
    return -(-n // _ALIGN) * _ALIGN


def _quantize_rows(w):
    w32 = w.float()
    s = w32.abs().amax(dim=1) / 127.0
    s = torch.where(s > 0, s, torch.ones_like(s))
    return (w32 / s[:, None]).round_().clamp_(-127, 127).to(torch.int8), s


class _Item:
    __slots__ = ("module", "attr", "shape", "dtype", "nbytes", "quant", "off", "raw_off")


class _Group:
    def __init__(self, block: nn.Module, skip=("adaln_proj",), codec=None):
        self.items = []
        off = raw = 0
        for mname, mod in block.named_modules():
            if any(mname == s or mname.startswith(s + ".") for s in skip):
                continue
            for pname, p in list(mod._parameters.items()):
                if p is None:
                    continue
                it = _Item()
                it.module, it.attr, it.shape, it.dtype = mod, pname, tuple(p.shape), p.dtype
                it.nbytes = p.numel() * p.element_size()
                it.quant = codec == "int8" and p.dim() == 2 and p.numel() >= 2 ** 16
                it.off, it.raw_off = off, raw
                off += _aligned(p.numel() + 4 * p.shape[0] if it.quant else it.nbytes)
                raw += _aligned(it.nbytes)
                self.items.append(it)
        self.nbytes, self.raw_bytes = off, raw

    def pack(self, flat):
        """Copy the module's current parameters into a stored-layout host buffer."""
        for it in self.items:
            p = it.module._parameters[it.attr].detach()
            if it.quant:
                q, s = _quantize_rows(p)
                n = p.numel()
                flat[it.off:it.off + n].view(torch.int8).copy_(q.reshape(-1).cpu())
                flat[it.off + n:it.off + n + 4 * it.shape[0]].view(torch.float32).copy_(s.cpu())
            else:
                flat[it.off:it.off + it.nbytes].view(it.dtype).copy_(p.reshape(-1).cpu())
        return flat

    def bind(self, slot, scratch):
        for it in self.items:
            if it.quant:
                n = it.shape[0] * it.shape[1]
                q = slot[it.off:it.off + n].view(torch.int8).view(it.shape)
                s = slot[it.off + n:it.off + n + 4 * it.shape[0]].view(torch.float32)
                w = scratch[it.raw_off:it.raw_off + it.nbytes].view(it.dtype).view(it.shape)
                w.copy_(q.float().mul_(s[:, None]))
            else:
                w = slot[it.off:it.off + it.nbytes].view(it.dtype).view(it.shape)
            it.module._parameters[it.attr] = nn.Parameter(w, requires_grad=False)

    def unbind(self):
        for it in self.items:
            it.module._parameters[it.attr] = nn.Parameter(torch.empty(it.shape, dtype=it.dtype, device="meta"),
                                                          requires_grad=False)


class BlockStreamer:
    """Streams the parameters of ``blocks`` through two GPU slots, one block ahead of compute."""

    def __init__(self, blocks, device, codec=None):
        self.blocks = list(blocks)
        if len(self.blocks) < 2:
            raise ValueError("need at least two streamed blocks")
        self.device = torch.device(device)
        if self.device.type == "cuda" and self.device.index is None:
            self.device = torch.device("cuda", torch.cuda.current_device())
        for b in self.blocks:  # buffers (LoRA masks, norm statistics) stay resident
            for m in b.modules():
                for k, buf in list(m._buffers.items()):
                    if buf is not None:
                        m._buffers[k] = buf.to(self.device)
        self.groups = [_Group(b, codec=codec) for b in self.blocks]
        self.host = [g.pack(torch.empty(g.nbytes, dtype=torch.uint8).pin_memory()) for g in self.groups]
        for g in self.groups:
            g.unbind()
        slot_bytes = max(g.nbytes for g in self.groups)
        self.slots = [torch.empty(slot_bytes, dtype=torch.uint8, device=self.device) for _ in range(2)]
        self.scratch = (torch.empty(max(g.raw_bytes for g in self.groups), dtype=torch.uint8, device=self.device)
                        if codec else None)
        self.stream = torch.cuda.Stream(device=self.device)
        self.compute_done = [torch.cuda.Event() for _ in range(2)]
        self.ready: dict = {}
        self.cond = threading.Condition()
        self.requests: queue.Queue = queue.Queue()
        self.error = None
        self.hooks = []
        for i, b in enumerate(self.blocks):
            self.hooks.append(b.register_forward_pre_hook(self._pre(i)))
            self.hooks.append(b.register_forward_hook(self._post(i)))
        self.bytes_per_pass = sum(g.nbytes for g in self.groups)
        self.worker = threading.Thread(target=self._run, daemon=True)
        self.worker.start()
        self.requests.put(0)
        self.requests.put(1)

    def _run(self):
        torch.cuda.set_device(self.device)
        try:
            while True:
                g = self.requests.get()
                if g is None:
                    return
                slot = g % 2
                n = self.groups[g].nbytes
                with torch.cuda.stream(self.stream):
                    self.stream.wait_event(self.compute_done[slot])
                    self.slots[slot][:n].copy_(self.host[g][:n], non_blocking=True)
                    ev = torch.cuda.Event()
                    ev.record(self.stream)
                with self.cond:
                    self.ready[g] = ev
                    self.cond.notify_all()
        except Exception as e:  # surfaced in the compute thread instead of hanging it
            with self.cond:
                self.error = e
                self.cond.notify_all()

    def _pre(self, i):
        def hook(module, args):
            with self.cond:
                while i not in self.ready and self.error is None:
                    self.cond.wait(timeout=60.0)
                    if i not in self.ready and self.error is None and not self.worker.is_alive():
                        self.error = RuntimeError("streaming worker died")
                if self.error is not None:
                    raise RuntimeError("weight streaming failed") from self.error
                ev = self.ready.pop(i)
            torch.cuda.current_stream().wait_event(ev)
            self.groups[i].bind(self.slots[i % 2], self.scratch)

        return hook

    def _post(self, i):
        def hook(module, args, output):
            self.compute_done[i % 2].record(torch.cuda.current_stream())
            self.groups[i].unbind()
            self.requests.put((i + 2) % len(self.groups))

        return hook

    def close(self):
        for h in self.hooks:
            h.remove()
        self.requests.put(None)
        self.worker.join(timeout=60)
        torch.cuda.synchronize(self.device)
        self.slots = self.scratch = self.host = None


class LowMemH3:
    """An ``H3Model`` (on the CPU) run with its blocks streamed; everything else resident.

    ``timesteps_per_step``: the distinct-timestep tensors the sampler will pass at each step, so the
    adaLN tables are built before sampling and the projections dropped."""

    def __init__(self, model, device, timesteps_per_step, codec=None):
        self.model = model.eval().requires_grad_(False)
        self.device = torch.device(device)
        if self.device.type == "cuda" and self.device.index is None:
            self.device = torch.device("cuda", torch.cuda.current_device())
        blocks = list(model.transformer_blocks)
        # resident pieces
        for name in ("proj_in", "audio_proj_in", "context_embedder", "time_embedder", "token_refiner", "norm_out",
                     "proj_out", "audio_proj_out"):
            getattr(model, name).to(self.device)
        # adaLN tables per step, one block's projection on the device at a time
        self.tables = [[None] * len(blocks) for _ in timesteps_per_step]
        with torch.no_grad():
            tembs = [model.temb(ts.to(self.device)) for ts in timesteps_per_step]
            for i, b in enumerate(blocks):
                b.adaln_proj.to(self.device)
                for s, temb in enumerate(tembs):
                    self.tables[s][i] = b.adaln_tables(temb)
                b.adaln_proj = None
        self.streamer = BlockStreamer(blocks, self.device, codec=codec)
        self._text_cache = []

    @torch.no_grad()
    def precompute_text(self, prompt_embeds_list):
        self._text_cache = [(pe, self.model.refine_text(pe.to(self.device))) for pe in prompt_embeds_list]
        self.model.token_refiner = None
        torch.cuda.empty_cache()

    def text_features(self, prompt_embeds):
        for known, out in self._text_cache:
            if known.shape == prompt_embeds.shape and torch.equal(known.cpu(), prompt_embeds.cpu()):
                return out
        raise RuntimeError("prompt not precomputed: call precompute_text with every prompt first")

    def close(self):
        self.streamer.close()
