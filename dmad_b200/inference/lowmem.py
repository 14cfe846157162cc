"""Low-VRAM inference: stream transformer blocks host -> device one layer ahead of compute.

Parity with dmad_h3/lowmem.py (ShardIndex :41-76, Streamer :176-331, LowMemTextEncoder :337-393,
AdaLNTables :400-413, _chunked_block_forward :416-461, TextLookup :464-475, LowMemTransformer :478-574):
* each block's weights (minus its adaLN projection) form one group with a fixed byte layout; the groups
  come from a tensor source: the memory-mapped safetensors shards of a checkpoint (``ShardIndex``) or
  the weights of a model already in host memory (``StateSource``);
* the bytes reach the GPU either from pinned host copies made once (``cache_in_ram``) or, per pass,
  from the source through two pinned staging buffers (host memory stays at two blocks);
* two rotating GPU slots; a worker thread issues ``cudaMemcpyAsync`` (``copy_(non_blocking=True)``) of
  block i+2 on a side stream once the compute stream has recorded that the slot's previous occupant is
  done; a forward pre-hook makes the compute stream wait on the copy and binds the parameters as views
  into the slot, the post-hook records ``compute_done`` and unbinds;
* the adaLN projections (the bulk of the parameters) depend only on the sampling step, so their outputs
  are tabulated per step up front and the projections are never streamed;
* the token refiner sees only the text, so its output is computed once per prompt;
* optional int8 per-output-row codec, dequantised to bf16 on the GPU right before use (changes the
  samples; off by default); streamed from disk it is written once to a cache directory validated by a
  manifest of the shards it came from;
* ``chunked_block_forward``: a block forward that holds at most ``rows`` rows of every intermediate
  except the keys and values (the attention still sees the whole sequence).
The kernels and their order are those of the resident model, so without the codec and the row chunking
the output is bit-identical to the resident run.  On a CPU device the same code runs with synchronous
copies (no streams or events), which is how the bookkeeping is tested without a GPU.
"""
from __future__ import annotations

import contextlib
import hashlib
import json
import queue
import threading
from pathlib import Path

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


# ----------------------------------------------------------------------------------------------- sources


class ShardIndex:
    """Tensor name -> shard of a safetensors directory (with or without an index file); shards are
    memory-mapped once touched, and ``tensor`` reads one entry."""

    def __init__(self, directory):
        from safetensors import safe_open

        self.directory = Path(directory).expanduser()
        self.where: dict = {}
        index = sorted(self.directory.glob("*.safetensors.index.json"))
        if index:
            for key, fname in json.load(open(index[0]))["weight_map"].items():
                self.where[key] = self.directory / fname
        else:
            for path in sorted(self.directory.glob("*.safetensors")):
                with safe_open(str(path), "pt") as f:
                    for key in f.keys():
                        self.where[key] = path
        if not self.where:
            raise FileNotFoundError(f"no safetensors in {self.directory}")
        self._open: dict = {}
        self._lock = threading.Lock()

    def _handle(self, path):
        from safetensors import safe_open

        with self._lock:
            h = self._open.get(path)
            if h is None:
                h = self._open[path] = safe_open(str(path), "pt")
            return h

    def keys(self):
        return self.where.keys()

    def __contains__(self, key):
        return key in self.where

    def tensor(self, key):
        return self._handle(self.where[key]).get_tensor(key)

    def files(self):
        return sorted(set(self.where.values()))


class StateSource:
    """An in-memory state dict (a model's own weights) as a tensor source."""

    def __init__(self, state):
        self.state = state

    def keys(self):
        return self.state.keys()

    def __contains__(self, key):
        return key in self.state

    def tensor(self, key):
        return self.state[key]

    def files(self):
        return []


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


# ----------------------------------------------------------------------------------------------- groups


def _param_pieces(module: nn.Module, prefix: str, source) -> dict:
    """id(parameter) -> [(source key, element offset, numel)]: the state-dict entries of ``module`` the
    source holds that are contiguous pieces of one parameter (a fused projection is stored as one entry
    per segment, each a row range of the fused weight)."""
    params = {id(p) for p in module.parameters()}
    pieces: dict = {}
    for key, t in module.state_dict(prefix=prefix, keep_vars=True).items():
        if key not in source:
            continue
        base = t if id(t) in params else getattr(t, "_base", None)
        if base is None or id(base) not in params or not t.is_contiguous():
            continue
        pieces.setdefault(id(base), []).append((key, t.storage_offset() - base.storage_offset(), t.numel()))
    return pieces


class _Item:
    __slots__ = ("module", "attr", "shape", "dtype", "numel", "nbytes", "quant", "off", "raw_off", "pieces")


class _Group:
    """The streamed parameters of one block in a fixed byte layout (each item 256-byte aligned; an int8
    item stores its rows then the fp32 row scales).  Parameters the source does not cover (adapters,
    for instance) stay resident."""

    def __init__(self, block: nn.Module, prefix: str, source, codec=None, skip=("adaln_proj",)):
        pieces = _param_pieces(block, prefix, source)
        self.items, self.resident = [], []
        off = raw = 0
        for mname, mod in block.named_modules():
            if any(mname == s or mname.startswith(s + ".") for s in skip):
                continue
            for pname, p in list(mod._parameters.items()):
                if p is None:
                    continue
                pc = pieces.get(id(p))
                if pc is None or sum(n for _, _, n in pc) != p.numel():
                    self.resident.append((mod, pname))
                    continue
                it = _Item()
                it.module, it.attr, it.shape, it.dtype = mod, pname, tuple(p.shape), p.dtype
                it.numel = p.numel()
                it.nbytes = p.numel() * p.element_size()
                it.quant = codec == "int8" and p.dim() == 2 and p.numel() >= 2 ** 16
                it.off, it.raw_off, it.pieces = off, raw, sorted(pc, key=lambda x: x[1])
                off += _aligned(p.numel() + 4 * p.shape[0] if it.quant else it.nbytes)
                raw += _aligned(it.nbytes)
                self.items.append(it)
        if not self.items:
            raise ValueError(f"no parameter of the block under {prefix!r} is in the weight source")
        self.nbytes, self.raw_bytes = off, raw

    def read(self, source, flat, quant_device="cpu"):
        """Fills ``flat`` (uint8, at least ``nbytes``) with this group in its stored layout."""
        with torch.no_grad():
            for it in self.items:
                if it.quant:
                    w = torch.empty(it.numel, dtype=it.dtype, device=quant_device)
                    for key, o, n in it.pieces:
                        w[o:o + n].copy_(source.tensor(key).reshape(-1))
                    q, s = _quantize_rows(w.view(it.shape))
                    flat[it.off:it.off + it.numel].view(torch.int8).copy_(q.reshape(-1))
                    flat[it.off + it.numel:it.off + it.numel + 4 * it.shape[0]].view(torch.float32).copy_(s)
                else:
                    dst = flat[it.off:it.off + it.nbytes].view(it.dtype)
                    for key, o, n in it.pieces:
                        dst[o:o + n].copy_(source.tensor(key).reshape(-1))
        return flat

    def bind(self, slot, scratch):
        for it in self.items:
            if it.quant:
                q = slot[it.off:it.off + it.numel].view(torch.int8).view(it.shape)
                s = slot[it.off + it.numel:it.off + it.numel + 4 * it.shape[0]].view(torch.float32)
                w = scratch[it.raw_off:it.raw_off + it.nbytes].view(it.dtype).view(it.shape)
                w.copy_(q.float().mul_(s[:, None]))
            else:
                w = slot[it.off:it.off + it.nbytes].view(it.dtype).view(it.shape)
            it.module._parameters[it.attr] = nn.Parameter(w, requires_grad=False)

    def unbind(self):
        for it in self.items:
            it.module._parameters[it.attr] = nn.Parameter(torch.empty(it.shape, dtype=it.dtype, device="meta"),
                                                          requires_grad=False)


# --------------------------------------------------------------------------------------------- streamer


class BlockStreamer:
    """Streams the parameters of ``blocks`` through two device slots, one block ahead of compute.

    ``source``/``prefixes``: where each block's weights come from (default: the blocks' own weights,
    which must then be real host tensors).  ``cache_in_ram``: pinned host copies made once, else read
    from the source on every pass through two pinned staging buffers.  ``codec="int8"`` without
    ``cache_in_ram`` needs ``cache_dir`` for the quantised copy."""

    def __init__(self, blocks, device, codec=None, source=None, prefixes=None, cache_in_ram=True, cache_dir=None,
                 log=None):
        self.blocks = list(blocks)
        if len(self.blocks) < 2:
            raise ValueError("need at least two streamed blocks")
        if codec not in (None, "int8"):
            raise ValueError(f"unknown weight codec {codec!r}")
        if codec is not None and not cache_in_ram and cache_dir is None:
            raise ValueError("int8 weights streamed from disk need a cache_dir for the quantised copy")
        self.device = torch.device(device)
        if self.device.type == "cuda" and self.device.index is None:
            self.device = torch.device("cuda", torch.cuda.current_device())
        self.cuda = self.device.type == "cuda"
        self.codec = codec
        if source is None:
            if any(p.device.type == "meta" for b in self.blocks for p in b.parameters()):
                raise ValueError("blocks on the meta device need a weight source (ShardIndex)")
            sources = [StateSource(b.state_dict()) for b in self.blocks]
            prefixes = [""] * len(self.blocks)
        else:
            sources = [source] * len(self.blocks)
            prefixes = list(prefixes)
        self.groups = [_Group(b, p, s, codec) for b, p, s in zip(self.blocks, prefixes, sources)]
        for b, g in zip(self.blocks, self.groups):  # adapters, norm statistics, masks stay resident
            for mod, name in g.resident:
                p = mod._parameters[name]
                if p.device.type == "meta":
                    raise ValueError(f"{type(mod).__name__}.{name} is neither in the weight source nor loaded")
                mod._parameters[name] = nn.Parameter(p.detach().to(self.device), requires_grad=False)
            _buffers_to(b, self.device)
        slot_bytes = max(g.nbytes for g in self.groups)
        self.bytes_per_pass = sum(g.nbytes for g in self.groups)
        self.sources, self.host, self.staging, self.cache_files = sources, None, None, None
        if cache_in_ram:
            self.host = []
            for i, g in enumerate(self.groups):
                self.host.append(g.read(sources[i], self._host_buffer(g.nbytes), self.device))
                if log and (i + 1) % 10 == 0:
                    log(f"cached {i + 1}/{len(self.groups)} blocks in host memory")
            self.sources = None  # the in-memory weights can go
        else:
            self.staging = [self._host_buffer(slot_bytes) for _ in range(2)]
            if codec is not None:
                self.cache_files = self._disk_cache(Path(cache_dir).expanduser(), sources, log)
        for g in self.groups:
            g.unbind()
        self.slots = [torch.empty(slot_bytes, dtype=torch.uint8, device=self.device) for _ in range(2)]
        self.scratch = (torch.empty(max(g.raw_bytes for g in self.groups), dtype=torch.uint8, device=self.device)
                        if codec else None)
        self.stream = torch.cuda.Stream(device=self.device) if self.cuda else None
        self.compute_done = [torch.cuda.Event() for _ in range(2)] if self.cuda else [None, None]
        self.staged = [None, None]  # per staging buffer: the event of the copy that last read it
        # the k-th requested group goes to slot k % 2 (groups are consumed in request order), so with an
        # odd block count the wrap-around from the last block to the first still alternates slots
        self.bound_slot = [0] * len(self.blocks)
        self.ready: dict = {}
        self.cond = threading.Condition()
        self.requests: queue.Queue = queue.Queue()
        self.error = None
        self.hooks = []
        for i, b in enumerate(self.blocks):
            self.hooks.append(b.register_forward_pre_hook(self._pre(i)))
            self.hooks.append(b.register_forward_hook(self._post(i)))
        self.worker = threading.Thread(target=self._run, daemon=True)
        self.worker.start()
        self.requests.put(0)
        self.requests.put(1)

    def _host_buffer(self, n):
        t = torch.empty(n, dtype=torch.uint8)
        return t.pin_memory() if self.cuda else t

    def _disk_cache(self, cache_dir, sources, log):
        """One file per group in the stored layout, written once and validated against a manifest of the
        shards it was built from (an in-memory source has no shards and is rewritten every time)."""
        cache_dir.mkdir(parents=True, exist_ok=True)
        shard_files = sources[0].files()
        manifest = {"codec": self.codec, "groups": [g.nbytes for g in self.groups],
                    "shards": [[p.name, p.stat().st_size] for p in shard_files]}
        files = [cache_dir / f"group_{i:03d}.bin" for i in range(len(self.groups))]
        mpath = cache_dir / "manifest.json"
        valid = (bool(shard_files) and mpath.is_file() and json.load(open(mpath)) == manifest
                 and all(f.is_file() and f.stat().st_size == g.nbytes for f, g in zip(files, self.groups)))
        if not valid:
            if log:
                log(f"writing the {self.codec} copy of the streamed weights to {cache_dir} (once)")
            if mpath.exists():
                mpath.unlink()
            for i, (f, g) in enumerate(zip(files, self.groups)):
                flat = g.read(sources[i], torch.zeros(g.nbytes, dtype=torch.uint8), self.device)
                with open(f, "wb") as h:
                    h.write(memoryview(flat.numpy()))
            json.dump(manifest, open(mpath, "w"))
        return files

    def _fill_staging(self, g, buf):
        if self.cache_files is not None:
            with open(self.cache_files[g], "rb") as h:
                h.readinto(memoryview(buf.numpy())[:self.groups[g].nbytes])
        else:
            self.groups[g].read(self.sources[g], buf, self.device)
        return buf

    def _run(self):
        if self.cuda:
            torch.cuda.set_device(self.device)
        seq = 0
        try:
            while True:
                g = self.requests.get()
                if g is None:
                    return
                slot = seq % 2
                seq += 1
                n = self.groups[g].nbytes
                if self.host is not None:
                    src = self.host[g]
                else:
                    if self.staged[slot] is not None:  # the copy that last read this staging buffer
                        self.staged[slot].synchronize()
                    src = self._fill_staging(g, self.staging[slot])
                ev = None
                if self.cuda:
                    with torch.cuda.stream(self.stream):
                        self.stream.wait_event(self.compute_done[slot])
                        self.slots[slot][:n].copy_(src[:n], non_blocking=True)
                        ev = torch.cuda.Event()
                        ev.record(self.stream)
                    if self.host is None:
                        self.staged[slot] = ev
                else:
                    self.slots[slot][:n].copy_(src[:n])
                with self.cond:
                    self.ready[g] = (ev, slot)
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
                ev, slot = self.ready.pop(i)
            if ev is not None:
                torch.cuda.current_stream(self.device).wait_event(ev)
            self.bound_slot[i] = slot
            self.groups[i].bind(self.slots[slot], self.scratch)

        return hook

    def _post(self, i):
        def hook(module, args, output):
            if self.cuda:
                self.compute_done[self.bound_slot[i]].record(torch.cuda.current_stream(self.device))
            self.groups[i].unbind()
            self.requests.put((i + 2) % len(self.groups))

        return hook

    def close(self):
        for h in self.hooks:
            h.remove()
        self.requests.put(None)
        self.worker.join(timeout=60)
        if self.cuda:
            torch.cuda.synchronize(self.device)
        self.slots = self.scratch = self.host = self.staging = self.sources = None


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

    def forward(h, tables, adaln_idx, cos, sin, cp=None, L_valid=None):
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
    """(H3Model, ShardIndex) for a transformer directory: the resident modules loaded on ``device``,
    the blocks left on the meta device for ``LowMemH3`` to stream from the shards."""
    from ..models.h3 import H3Model
    from .h3 import config_from_transformer_dir, resolve_transformer_dir

    root = resolve_transformer_dir(model_dir)
    with torch.device("meta"):
        model = H3Model(config_from_transformer_dir(root)).to(dtype)
    source = ShardIndex(root)
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
    holds real weights in host memory; with a ``ShardIndex`` (``build_streamed_h3``) its blocks are on
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
        self.streamer = BlockStreamer(blocks, self.device, codec=codec, source=source, prefixes=prefixes,
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
        self.source = ShardIndex(tdir)
        names = {id(m): n for n, m in model.named_modules()}
        lm_prefix = names[id(self.lm)] + "."
        emb = self.lm.embed_tokens
        load_resident(emb, lm_prefix + "embed_tokens.", self.source, self.device)
        self.streamer = BlockStreamer(list(self.lm.layers), self.device, source=self.source,
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
