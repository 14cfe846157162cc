"""Low-VRAM inference: the transformer's repeated blocks stream host -> device while the GPU computes.

What it reproduces (dmad_h3/lowmem.py: the ``--low-vram`` path of the H3 CLI): the blocks' weights
stay on the host and only a few blocks' worth of device memory holds them, one block ahead of compute,
with the sampled output bit-identical to the resident run; optional int8 weights; the adaLN
projections tabulated per sampling step instead of streamed; the text refiner run once per prompt; a
row-chunked block forward; the Qwen3-VL text encoder streamed layer by layer.

How (this library's design):
* ``SafetensorsCatalog`` parses the shards' headers itself, so every tensor is a (file, byte offset,
  length) triple.  A block whose stored dtypes match the model's streams straight from those byte
  ranges: the native engine ``pread``s them into a pinned staging buffer, no Python on the path.
* ``BlockLayout`` packs one block's streamed parameters into a fixed byte layout (each 256-byte
  aligned; fused projections stored as several checkpoint entries map to several extents of one
  parameter) and knows where every byte comes from.
* ``LayerStreamer`` drives the native engine ``dmad_b200._C.H2DStreamer`` (csrc/h2d_stream.cpp): K
  device slots, one copy stream, events, a C++ worker thread issuing ``cudaMemcpyAsync`` from pinned
  memory on the side stream.  A forward pre-hook ``acquire``s the block's slot (the compute stream waits
  on the copy's event, never the host on the GPU) and binds the parameters as views into it; the post-
  hook unbinds and ``release``s, which queues the block K positions later in the cyclic schedule.
* Groups come from pinned RAM copies made once (``cache_in_ram``), straight from the shards, or from an
  int8 cache directory (one file per block, per-output-row absmax scales, checked against a
  fingerprint of the shards it was made from).
On a CPU device the engine runs the same schedule with synchronous memcpy into host slots, which is
how the bookkeeping is tested without a GPU.
"""
from __future__ import annotations

import contextlib
import hashlib
import json
import mmap
import os
import struct
from pathlib import Path

import torch
import torch.nn as nn

_ALIGN = 256
_ST_DTYPES = {"BF16": torch.bfloat16, "F16": torch.float16, "F32": torch.float32, "F64": torch.float64,
              "I64": torch.int64, "I32": torch.int32, "I16": torch.int16, "I8": torch.int8, "U8": torch.uint8,
              "BOOL": torch.bool}


def _round_up(n: int) -> int:
    return (n + _ALIGN - 1) // _ALIGN * _ALIGN


def int8_rows(w: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Symmetric per-output-row int8 code: q = round(w / s), s = max|w_row| / 127 (s = 1 for a zero row)."""
    w32 = w.float()
    scale = w32.abs().amax(dim=1).div(127.0)
    scale = scale.masked_fill(scale == 0, 1.0)
    return torch.clamp(torch.round(w32 / scale.unsqueeze(1)), -127, 127).to(torch.int8), scale


# ----------------------------------------------------------------------------------------------- weights on disk


class SafetensorsCatalog:
    """Every tensor of a directory of ``*.safetensors`` shards as (file, byte offset, length, dtype, shape),
    read from the shards' own headers (8-byte little-endian header length, then a JSON table of
    ``dtype`` / ``shape`` / ``data_offsets`` relative to the end of the header)."""

    def __init__(self, directory):
        self.directory = Path(directory).expanduser()
        self.entries: dict = {}
        self.shards = sorted(self.directory.glob("*.safetensors"))
        for path in self.shards:
            with open(path, "rb") as f:
                (hlen,) = struct.unpack("<Q", f.read(8))
                header = json.loads(f.read(hlen))
            base = 8 + hlen
            for key, meta in header.items():
                if key == "__metadata__":
                    continue
                start, end = meta["data_offsets"]
                dtype = _ST_DTYPES.get(meta["dtype"])
                if dtype is None:
                    raise ValueError(f"{path.name}: tensor {key} has unsupported dtype {meta['dtype']}")
                self.entries[key] = (path, base + int(start), int(end) - int(start), dtype, tuple(meta["shape"]))
        if not self.entries:
            raise FileNotFoundError(f"{self.directory}: no tensors found in *.safetensors files")
        self._maps: dict = {}

    def keys(self):
        return self.entries.keys()

    def __contains__(self, key):
        return key in self.entries

    def location(self, key):
        """(path, byte offset, byte length, dtype, shape) of one tensor."""
        return self.entries[key]

    def tensor(self, key) -> torch.Tensor:
        """A read-only CPU view of one tensor over the memory-mapped shard."""
        path, off, n, dtype, shape = self.entries[key]
        mm = self._maps.get(path)
        if mm is None:
            with open(path, "rb") as f:
                mm = self._maps[path] = mmap.mmap(f.fileno(), 0, access=mmap.ACCESS_READ)
        if n == 0:
            return torch.empty(shape, dtype=dtype)
        import warnings
        with warnings.catch_warnings():
            warnings.simplefilter("ignore")  # the view is read-only; callers copy out of it
            raw = torch.frombuffer(mm, dtype=torch.uint8, count=n, offset=off)
        return raw.view(dtype).reshape(shape)

    def fingerprint(self) -> list:
        return [[p.name, p.stat().st_size, p.stat().st_mtime_ns] for p in self.shards]


class _DictSource:
    """A state dict held in memory, behind the same ``keys`` / ``tensor`` interface."""

    def __init__(self, state):
        self.state = state

    def keys(self):
        return self.state.keys()

    def __contains__(self, key):
        return key in self.state

    def tensor(self, key):
        return self.state[key]


@contextlib.contextmanager
def empty_parameters():
    """Modules built inside get their parameters on the meta device (no memory, no init cost) while
    buffers stay real, so computed buffers (rotary frequencies and the like) survive."""
    orig = nn.Module.register_parameter

    def register(self, name, param):
        orig(self, name, param)
        p = self._parameters.get(name)
        if p is not None and p.device.type != "meta":
            self._parameters[name] = nn.Parameter(p.detach().to("meta"), requires_grad=p.requires_grad)

    nn.Module.register_parameter = register
    try:
        yield
    finally:
        nn.Module.register_parameter = orig


def load_resident(module: nn.Module, prefix: str, source, device, dtype=None):
    """Materialises ``module`` on ``device`` from the source entries under ``prefix`` (strict)."""
    sd = {k[len(prefix):]: source.tensor(k) for k in source.keys() if k.startswith(prefix)}
    if dtype is not None:
        module.to(dtype)
    module.to_empty(device=device)
    with torch.no_grad():
        module.load_state_dict(sd, strict=True)
    return module


def _buffers_to(module: nn.Module, device):
    for m in module.modules():
        for k, buf in list(m._buffers.items()):
            if buf is not None and buf.device.type != "meta":
                m._buffers[k] = buf.to(device)


# ----------------------------------------------------------------------------------------------- block layout


class _Param:
    __slots__ = ("module", "name", "shape", "dtype", "numel", "nbytes", "int8", "offset", "wide_offset", "parts")


class BlockLayout:
    """One block's streamed parameters in a fixed byte layout, and where each byte comes from.

    ``parts`` of a parameter: (source key, element offset in the parameter, element count), because a
    checkpoint may store one fused parameter as several entries (the q / k / v rows of a fused
    projection are views of one weight).  An int8 parameter stores its rows, then its fp32 row scales;
    ``wide_offset`` is its place in the bf16 scratch it is decoded into.  Parameters the source does not
    cover (adapters) stay resident."""

    def __init__(self, block: nn.Module, prefix: str, source, int8: bool = False, skip=("adaln_proj",)):
        owner = {id(p): (m, n) for m in block.modules() for n, p in m._parameters.items() if p is not None}
        skipped = {id(p) for s in skip if hasattr(block, s) and getattr(block, s) is not None
                   for p in getattr(block, s).parameters()}
        parts: dict = {}
        for key, t in block.state_dict(prefix=prefix, keep_vars=True).items():
            base = t if id(t) in owner else t._base
            if key in source and base is not None and id(base) in owner and t.is_contiguous():
                parts.setdefault(id(base), []).append((key, t.storage_offset() - base.storage_offset(), t.numel()))
        self.params, self.resident = [], []
        cursor = wide = 0
        for pid, (mod, name) in owner.items():
            if pid in skipped:
                continue
            p = mod._parameters[name]
            pc = sorted(parts.get(pid, []), key=lambda x: x[1])
            if sum(n for _, _, n in pc) != p.numel():
                self.resident.append((mod, name))
                continue
            it = _Param()
            it.module, it.name, it.shape, it.dtype, it.numel = mod, name, tuple(p.shape), p.dtype, p.numel()
            it.nbytes = p.numel() * p.element_size()
            it.int8 = bool(int8) and p.dim() == 2 and p.numel() >= 1 << 16
            it.offset, it.wide_offset, it.parts = cursor, wide, pc
            cursor += _round_up(it.numel + 4 * it.shape[0] if it.int8 else it.nbytes)
            wide += _round_up(it.nbytes)
            self.params.append(it)
        if not self.params:
            raise ValueError(f"block {prefix!r}: none of its parameters is in the weight source")
        self.nbytes, self.wide_bytes = cursor, wide
        self.int8 = any(it.int8 for it in self.params)

    def file_extents(self, catalog: SafetensorsCatalog):
        """[(path, file offset, bytes, layout offset)] when every byte can be read from the shards as stored
        (no int8 code, stored dtype = parameter dtype), else None."""
        if self.int8 or not isinstance(catalog, SafetensorsCatalog):
            return None
        out = []
        for it in self.params:
            esz = it.nbytes // it.numel
            for key, elem_off, n in it.parts:
                path, off, nbytes, dtype, _ = catalog.location(key)
                if dtype != it.dtype or nbytes != n * esz:
                    return None
                out.append((path, off, nbytes, it.offset + elem_off * esz))
        return out

    @torch.no_grad()
    def pack(self, source, out: torch.Tensor, work_device="cpu") -> torch.Tensor:
        """Writes the layout into ``out`` (uint8, at least ``nbytes``); int8 coding runs on ``work_device``."""
        for it in self.params:
            if it.int8:
                w = torch.empty(it.numel, dtype=it.dtype, device=work_device)
                for key, o, n in it.parts:
                    w[o:o + n].copy_(source.tensor(key).reshape(-1))
                q, scale = int8_rows(w.view(it.shape))
                out[it.offset:it.offset + it.numel].view(torch.int8).copy_(q.reshape(-1))
                out[it.offset + it.numel:it.offset + it.numel + 4 * it.shape[0]].view(torch.float32).copy_(scale)
            else:
                dst = out[it.offset:it.offset + it.nbytes].view(it.dtype)
                for key, o, n in it.parts:
                    dst[o:o + n].copy_(source.tensor(key).reshape(-1))
        return out

    def attach(self, slot: torch.Tensor, wide: torch.Tensor | None):
        """Points the block's parameters at their bytes in ``slot`` (int8 ones decoded into ``wide``)."""
        for it in self.params:
            if it.int8:
                q = slot[it.offset:it.offset + it.numel].view(torch.int8).view(it.shape)
                scale = slot[it.offset + it.numel:it.offset + it.numel + 4 * it.shape[0]].view(torch.float32)
                w = wide[it.wide_offset:it.wide_offset + it.nbytes].view(it.dtype).view(it.shape)
                w.copy_(q.float().mul_(scale.unsqueeze(1)))
            else:
                w = slot[it.offset:it.offset + it.nbytes].view(it.dtype).view(it.shape)
            it.module._parameters[it.name] = nn.Parameter(w, requires_grad=False)

    def detach(self):
        for it in self.params:
            it.module._parameters[it.name] = nn.Parameter(torch.empty(it.shape, dtype=it.dtype, device="meta"),
                                                          requires_grad=False)


# --------------------------------------------------------------------------------------------- streamer


class LayerStreamer:
    """Streams the parameters of ``blocks`` through ``slots`` device buffers in the blocks' order.

    ``source`` / ``prefixes``: where each block's weights come from (default: the blocks' own weights,
    which must then be real host tensors).  ``cache_in_ram``: pinned host copies made once; otherwise
    every pass reads the shards (or the int8 cache directory) through two pinned staging buffers, so
    host memory holds two blocks.  ``codec="int8"`` without ``cache_in_ram`` needs ``cache_dir``."""

    def __init__(self, blocks, device, codec=None, source=None, prefixes=None, cache_in_ram=True, cache_dir=None,
                 slots: int = 2, timeout_s: float = 600.0, log=None):
        from .. import ops

        self.blocks = list(blocks)
        if len(self.blocks) < 2:
            raise ValueError("layer streaming needs at least two blocks")
        if codec not in (None, "int8"):
            raise ValueError(f"weight codec must be None or 'int8', not {codec!r}")
        if codec and not cache_in_ram and cache_dir is None:
            raise ValueError("int8 weights read from disk on every pass are read from a cache directory of the "
                             "coded weights: pass cache_dir (or cache_in_ram=True)")
        self.device = torch.device(device)
        if self.device.type == "cuda" and self.device.index is None:
            self.device = torch.device("cuda", torch.cuda.current_device())
        self.cuda = self.device.type == "cuda"
        self.codec = codec
        if source is None:
            if any(p.device.type == "meta" for b in self.blocks for p in b.parameters()):
                raise ValueError("blocks whose weights are on the meta device need a weight source "
                                 "(a SafetensorsCatalog of the checkpoint)")
            sources = [_DictSource(b.state_dict()) for b in self.blocks]
            prefixes = [""] * len(self.blocks)
        else:
            sources = [source] * len(self.blocks)
            prefixes = list(prefixes)
        self.layouts = [BlockLayout(b, p, s, int8=codec == "int8") for b, p, s in zip(self.blocks, prefixes, sources)]
        for b, lay in zip(self.blocks, self.layouts):  # adapters and buffers stay on the device
            for mod, name in lay.resident:
                p = mod._parameters[name]
                if p.device.type == "meta":
                    raise ValueError(f"{type(mod).__name__}.{name}: not in the weight source and never loaded")
                mod._parameters[name] = nn.Parameter(p.detach().to(self.device), requires_grad=False)
            _buffers_to(b, self.device)
        slot_bytes = max(lay.nbytes for lay in self.layouts)
        self.bytes_per_pass = sum(lay.nbytes for lay in self.layouts)
        self.host = None       # pinned RAM copies (cache_in_ram)
        self.staging = []      # pinned staging buffers (groups read from files)
        self.engine = ops.ext().H2DStreamer  # fails loudly without the native extension
        extents = [None] * len(self.layouts)
        if source is None:
            cache_in_ram = True  # the weights are in host memory already
        if not cache_in_ram and not codec:
            extents = [lay.file_extents(src) for lay, src in zip(self.layouts, sources)]
        if cache_in_ram:
            self.host = []
            for i, lay in enumerate(self.layouts):
                self.host.append(lay.pack(sources[i], self._host_bytes(lay.nbytes), self.device))
                if log and (i + 1) % 10 == 0:
                    log(f"{i + 1} of {len(self.layouts)} blocks copied to pinned host memory")
        elif codec or any(e is None for e in extents):
            # int8 code, or stored dtypes that differ from the model's: a converted copy on disk, made once
            kind = codec or "converted"
            where = Path(cache_dir).expanduser() if cache_dir else default_cache_dir(sources[0].directory, kind)
            files = self._disk_copy(where, kind, sources, log)
            extents = [[(str(f), 0, lay.nbytes, 0)] for f, lay in zip(files, self.layouts)]
        for lay in self.layouts:
            lay.detach()
        self.slots = [torch.empty(slot_bytes, dtype=torch.uint8, device=self.device) for _ in range(int(slots))]
        self.wide = (torch.empty(max(lay.wide_bytes for lay in self.layouts), dtype=torch.uint8, device=self.device)
                     if codec else None)
        if self.host is None:
            self.staging = [self._host_bytes(slot_bytes) for _ in range(2)]
        self.native = self.engine([t.data_ptr() for t in self.slots], slot_bytes,
                                  self.device.index if self.cuda else -1,
                                  [t.data_ptr() for t in self.staging], slot_bytes if self.staging else 0,
                                  float(timeout_s))
        file_ids: dict = {}
        for i, lay in enumerate(self.layouts):
            if self.host is not None:
                self.native.add_ram_group(self.host[i].data_ptr(), lay.nbytes)
            else:
                ext = []
                for path, off, n, dst in extents[i]:
                    if path not in file_ids:
                        file_ids[str(path)] = self.native.add_file(str(path))
                    ext.append([file_ids[str(path)], int(off), int(n), int(dst)])
                self.native.add_file_group(ext, lay.nbytes)
        self.hooks = []
        for i, b in enumerate(self.blocks):
            self.hooks.append(b.register_forward_pre_hook(self._before(i)))
            self.hooks.append(b.register_forward_hook(self._after(i)))
        self.native.start(list(range(len(self.blocks))))

    # a copy of the blocks in their streamed layout (int8-coded or dtype-converted): one file per block,
    # reused while the shards' fingerprint is unchanged
    def _disk_copy(self, cache_dir: Path, kind: str, sources, log):
        cache_dir.mkdir(parents=True, exist_ok=True)
        catalog = sources[0] if isinstance(sources[0], SafetensorsCatalog) else None
        stamp = {"format": f"dmad_b200 {kind} layout v1", "blocks": [lay.nbytes for lay in self.layouts],
                 "dtypes": sorted({str(it.dtype) for lay in self.layouts for it in lay.params}),
                 "source": catalog.fingerprint() if catalog else None}
        files = [cache_dir / f"block{i:04d}.bin" for i in range(len(self.layouts))]
        index = cache_dir / "index.json"
        reuse = (catalog is not None and index.is_file() and json.loads(index.read_text()) == stamp
                 and all(f.is_file() and f.stat().st_size == lay.nbytes for f, lay in zip(files, self.layouts)))
        if not reuse:
            if log:
                log(f"writing the {kind} layout of {len(files)} blocks to {cache_dir}; later runs reuse it")
            index.unlink(missing_ok=True)
            for i, (f, lay) in enumerate(zip(files, self.layouts)):
                buf = lay.pack(sources[i], torch.zeros(lay.nbytes, dtype=torch.uint8), self.device)
                tmp = f.with_suffix(".tmp")
                with open(tmp, "wb") as h:
                    h.write(buf.numpy().tobytes())
                os.replace(tmp, f)
            index.write_text(json.dumps(stamp))
        return files

    def _host_bytes(self, n):
        t = torch.empty(n, dtype=torch.uint8)
        return t.pin_memory() if self.cuda else t

    def _stream_handle(self):
        return torch.cuda.current_stream(self.device).cuda_stream if self.cuda else 0

    def _before(self, i):
        def hook(module, args):
            slot, group = self.native.acquire(self._stream_handle())
            if group != i:
                raise RuntimeError(f"layer streaming: block {i} ran where the schedule expected block {group} "
                                   f"(blocks must run in order, every pass)")
            self.layouts[i].attach(self.slots[slot], self.wide)

        return hook

    def _after(self, i):
        def hook(module, args, output):
            self.layouts[i].detach()
            self.native.release(self._stream_handle())

        return hook

    def stats(self) -> dict:
        return dict(self.native.stats())

    def close(self):
        for h in self.hooks:
            h.remove()
        self.hooks = []
        if self.native is not None:
            self.native.close()
        if self.cuda:
            torch.cuda.synchronize(self.device)
        self.native = None
        self.slots = self.wide = self.host = self.staging = None


# ------------------------------------------------------------------------------------ row-chunked block


def chunked_block_forward(block, rows: int):
    """An ``H3Block.forward`` that holds at most ``rows`` rows of every intermediate except k and v.

    Norms, modulation, projections, RoPE and the feed-forward are per row, so they run chunk by chunk
    and the residual stream is updated in place; k and v are built for the whole sequence first, and
    each chunk's queries are computed (from rows not yet updated) right before its attention.  The
    same ops as the resident forward on smaller matrices, so results can differ in the last bits."""
    from .. import ops

    attn, ff, eps = block.attn, block.ff, block.cfg.eps
    H, hd = attn.heads, attn.head_dim
    D = H * hd
    to_out = getattr(attn.to_out, "0")

    def forward(h, tables, adaln_idx, cos, sin, cp=None, L_valid=None, temb=None):
        if tables is None:
            tables = block.adaln_tables(temb)
        if cp is not None or not block.modulated:
            raise NotImplementedError("row chunking runs the modulated blocks of a single-GPU forward")
        sh1, sc1, g1, sh2, sc2, g2 = tables
        L = h.shape[0]
        size = -(-L // -(-L // rows))  # equal chunks of at most `rows` rows
        spans = [(s, min(s + size, L)) for s in range(0, L, size)]

        def modulated(s, e):
            return ops.ln_mod(h[s:e], sc1, sh1, a_add=1.0, gidx=adaln_idx[s:e], eps=eps)

        k, v = h.new_empty(L, D), h.new_empty(L, D)
        for s, e in spans:
            kv = attn.qkv.forward_rows(modulated(s, e), D, 3 * D)
            kk = ops.rms_norm(kv[:, :D].reshape((e - s) * H, hd), attn.norm_k.weight, eps).reshape(e - s, D)
            k[s:e] = ops.rope(kk, cos[s:e], sin[s:e], hd) if cos is not None else kk
            v[s:e] = kv[:, D:]
        for s, e in spans:
            q = attn.qkv.forward_rows(modulated(s, e), 0, D)
            q = ops.rms_norm(q.reshape((e - s) * H, hd), attn.norm_q.weight, eps).reshape(e - s, D)
            if cos is not None:
                q = ops.rope(q, cos[s:e], sin[s:e], hd)
            o = ops.flash_attention(q.view(1, e - s, H, hd), k.view(1, L, H, hd), v.view(1, L, H, hd))
            h[s:e] = ops.gate_residual(h[s:e], to_out(o.reshape(e - s, D)), g1, gidx=adaln_idx[s:e])
        del k, v
        for s, e in spans:
            x = ops.ln_mod(h[s:e], sc2, sh2, a_add=1.0, gidx=adaln_idx[s:e], eps=eps)
            h[s:e] = ops.gate_residual(h[s:e], ff(x), g2, gidx=adaln_idx[s:e])
        return h

    return forward


# ----------------------------------------------------------------------------------------- H3 transformer

_H3_RESIDENT = ("proj_in", "audio_proj_in", "context_embedder", "time_embedder", "token_refiner", "norm_out",
                "proj_out", "audio_proj_out")


def build_streamed_h3(model_dir, device, dtype=torch.bfloat16):
    """(H3Model, SafetensorsCatalog) for a transformer directory: the resident modules loaded on ``device``,
    the blocks left on the meta device for ``LowMemH3`` to stream from the shards."""
    from ..models.h3 import H3Model
    from .h3 import config_from_transformer_dir, resolve_transformer_dir

    root = resolve_transformer_dir(model_dir)
    with torch.device("meta"):
        model = H3Model(config_from_transformer_dir(root)).to(dtype)
    source = SafetensorsCatalog(root)
    for name in _H3_RESIDENT:
        load_resident(getattr(model, name), name + ".", source, device)
    return model.eval().requires_grad_(False), source


def default_cache_dir(model_dir, codec="int8") -> Path:
    key = hashlib.sha1(str(Path(model_dir).expanduser().resolve()).encode()).hexdigest()[:12]
    return Path.home() / ".cache" / "dmad_b200" / key / codec


class LowMemH3:
    """An ``H3Model`` run with its blocks streamed; everything else resident on ``device``.

    ``timesteps_per_step``: the distinct-timestep tensors the sampler will pass at each step, so the
    adaLN tables are built before sampling and the projections dropped.  Without ``source`` the model
    holds real weights in host memory; with a ``SafetensorsCatalog`` (``build_streamed_h3``) its blocks are on
    the meta device and read from the shards (adaLN projections one block at a time)."""

    def __init__(self, model, device, timesteps_per_step, codec=None, source=None, cache_in_ram=True, cache_dir=None,
                 chunk_rows=None, log=None):
        self.model = model.eval().requires_grad_(False)
        self.device = torch.device(device)
        if self.device.type == "cuda" and self.device.index is None:
            self.device = torch.device("cuda", torch.cuda.current_device())
        blocks = list(model.transformer_blocks)
        for name in _H3_RESIDENT:
            getattr(model, name).to(self.device)
        # adaLN tables per step, one block's projection on the device at a time
        self.tables = [[None] * len(blocks) for _ in timesteps_per_step]
        with torch.no_grad():
            tembs = [model.temb(ts.to(self.device)) for ts in timesteps_per_step]
            for i, b in enumerate(blocks):
                if source is not None and b.adaln_proj.weight.device.type == "meta":
                    load_resident(b.adaln_proj, f"transformer_blocks.{i}.adaln_proj.", source, self.device)
                else:
                    b.adaln_proj.to(self.device)
                for s, temb in enumerate(tembs):
                    self.tables[s][i] = b.adaln_tables(temb)
                b.adaln_proj = None
        if chunk_rows:
            for b in blocks:
                b.forward = chunked_block_forward(b, int(chunk_rows))
        prefixes = [f"transformer_blocks.{i}." for i in range(len(blocks))] if source is not None else None
        self.streamer = LayerStreamer(blocks, self.device, codec=codec, source=source, prefixes=prefixes,
                                      cache_in_ram=cache_in_ram, cache_dir=cache_dir, log=log)
        self._text_cache = []

    @torch.no_grad()
    def precompute_text(self, prompt_embeds_list):
        self._text_cache = [(pe, self.model.refine_text(pe.to(self.device))) for pe in prompt_embeds_list]
        self.model.token_refiner = None
        if self.device.type == "cuda":
            torch.cuda.empty_cache()

    def text_features(self, prompt_embeds):
        for known, out in self._text_cache:
            if known.shape == prompt_embeds.shape and torch.equal(known.cpu(), prompt_embeds.cpu()):
                return out
        raise RuntimeError("prompt not precomputed: call precompute_text with every prompt first")

    def close(self):
        self.streamer.close()


# ----------------------------------------------------------------------------------------- text encoder


class LowMemTextEncoder:
    """The H3 conditioner (a Qwen3-VL language model read at hidden layer ``layer``) with only the token
    embedding resident and the decoder layers streamed from the checkpoint's shards; the layers above
    the one read, the vision tower and the LM head are never materialised.

    ``encode`` returns what ``Qwen3VLConditioner.encode`` returns for the same checkpoint."""

    def __init__(self, model_dir, device, layer: int = 50, dtype=torch.bfloat16, cache_in_ram=False, log=None,
                 tokenizer=None, processor=None):
        from transformers import AutoConfig, AutoTokenizer, Qwen3VLForConditionalGeneration

        from .text_encoder import TEXT_TAG, _language_model

        root = Path(model_dir).expanduser()
        tdir = root / "text_encoder"
        self.device, self.layer, self.text_tag = torch.device(device), int(layer), TEXT_TAG
        config = AutoConfig.from_pretrained(str(tdir), local_files_only=True)
        with empty_parameters():
            try:
                model = Qwen3VLForConditionalGeneration._from_config(config, dtype=dtype)
            except TypeError:
                model = Qwen3VLForConditionalGeneration._from_config(config, torch_dtype=dtype)
        self.model = model.eval().requires_grad_(False)
        self.inner, self.lm = _language_model(model)
        if self.layer > len(self.lm.layers):
            raise ValueError(f"hidden layer {self.layer} outside 0..{len(self.lm.layers)}")
        self.lm.layers = nn.ModuleList(list(self.lm.layers)[:self.layer])
        self.lm.norm = nn.Identity()
        _buffers_to(self.model, self.device)
        self.source = SafetensorsCatalog(tdir)
        names = {id(m): n for n, m in model.named_modules()}
        lm_prefix = names[id(self.lm)] + "."
        emb = self.lm.embed_tokens
        load_resident(emb, lm_prefix + "embed_tokens.", self.source, self.device)
        self.streamer = LayerStreamer(list(self.lm.layers), self.device, source=self.source,
                                      prefixes=[f"{lm_prefix}layers.{i}." for i in range(len(self.lm.layers))],
                                      cache_in_ram=cache_in_ram, log=log)
        self.tokenizer = tokenizer or AutoTokenizer.from_pretrained(str(root / "tokenizer"), local_files_only=True)
        self.processor = processor
        if processor is None and tokenizer is None and (root / "processor").exists():
            from transformers import AutoProcessor
            self.processor = AutoProcessor.from_pretrained(str(root / "processor"), local_files_only=True)

    def inputs(self, prompt: str):
        ids = self.tokenizer(prompt, add_special_tokens=False)["input_ids"]
        if not ids:
            raise ValueError("the tokenizer produced no tokens for a non-empty prompt")
        input_ids = torch.tensor([list(ids)], dtype=torch.long, device=self.device)
        if self.processor is not None and hasattr(self.processor, "create_mm_token_type_ids"):
            mm = torch.tensor(self.processor.create_mm_token_type_ids([list(ids)]), dtype=torch.long,
                              device=self.device)
        else:
            mm = torch.zeros_like(input_ids)
        return input_ids, mm

    @torch.inference_mode()
    def encode(self, prompt: str, output_dtype=torch.bfloat16) -> dict:
        input_ids, mm = self.inputs(prompt)
        out = self.inner(input_ids=input_ids, attention_mask=torch.ones_like(input_ids), mm_token_type_ids=mm,
                         pixel_values=None, image_grid_thw=None, use_cache=False)
        emb = out.last_hidden_state.to(output_dtype).cpu()
        return {"prompt_embeds": emb,
                "text_token_tags": torch.full((input_ids.shape[1],), self.text_tag, dtype=torch.long)}

    def encode_all(self, prompts) -> list[dict]:
        return [self.encode(p) for p in prompts]

    def close(self):
        self.streamer.close()
        self.model = self.inner = self.lm = self.source = None
        if self.device.type == "cuda":
            torch.cuda.empty_cache()
