"""DMAD student LoRAs in the Diffusers safetensors layout.

File format (parity with dmad_h3/lora.py:23-75): per adapted module ``<module>.lora.down.weight`` = A
``[rank, in]`` and ``<module>.lora.up.weight`` = B ``[out, rank]``; the adapter adds ``(alpha/rank) B A x``;
alpha comes from the ``lora_alpha`` metadata entry, else equals the rank.  PEFT-style keys
(``lora_A`` / ``lora_B``, ``.default``, ``transformer.`` prefix) are accepted on read.

Module names are those of the model's reference layout (``transformer_blocks.3.attn.to_q``,
``blocks.0.self_attn.q``...).  Fused projections (q/k/v in one SegLinear) map each segment to its own
module name, so files round-trip with the reference's unfused layout.
"""
from __future__ import annotations

import torch
import torch.nn as nn

from .models.layers import SegLinear

_SUFFIXES = {
    ".lora.down.weight": "A",
    ".lora.up.weight": "B",
    ".lora_A.weight": "A",
    ".lora_B.weight": "B",
    ".lora_A.default.weight": "A",
    ".lora_B.default.weight": "B",
}


def read_lora_file(path):
    """-> (pairs, metadata), pairs: module name -> {"A": tensor, "B": tensor}."""
    from safetensors import safe_open

    pairs, meta = {}, {}
    with safe_open(str(path), "pt") as f:
        meta = dict(f.metadata() or {})
        for key in f.keys():
            for suffix, part in _SUFFIXES.items():
                if key.endswith(suffix):
                    mod = key[: -len(suffix)]
                    if mod.startswith("transformer."):
                        mod = mod[len("transformer."):]
                    pairs.setdefault(mod, {})[part] = f.get_tensor(key)
                    break
            else:
                raise ValueError(f"unexpected tensor in LoRA file: {key}")
    if not pairs:
        raise ValueError(f"no LoRA pairs in {path}")
    bad = [m for m, p in pairs.items() if set(p) != {"A", "B"}]
    if bad:
        raise ValueError(f"LoRA modules missing A or B: {bad[:5]}")
    return pairs, meta


def lora_rank_alpha(pairs, meta, alpha=None):
    ranks = {p["A"].shape[0] for p in pairs.values()}
    if len(ranks) != 1:
        raise ValueError(f"mixed LoRA ranks {sorted(ranks)}")
    rank = ranks.pop()
    if alpha is None:
        alpha = float(meta["lora_alpha"]) if "lora_alpha" in meta else float(rank)
    return rank, float(alpha)


def save_lora_file(path, pairs, rank, alpha, metadata=None):
    from safetensors.torch import save_file

    tensors = {}
    for mod, p in sorted(pairs.items()):
        tensors[f"{mod}.lora.down.weight"] = p["A"].contiguous()
        tensors[f"{mod}.lora.up.weight"] = p["B"].contiguous()
    meta = {"format": "pt", "lora_rank": str(rank), "lora_alpha": str(float(alpha))}
    meta.update(metadata or {})
    save_file(tensors, str(path), metadata=meta)


def _segment_module_names(model: nn.Module):
    """Yield (module name, SegLinear, segment name) with the reference's per-segment module names."""
    for name, mod in model.named_modules():
        if not isinstance(mod, SegLinear):
            continue
        parent = name.rsplit(".", 1)[0] if "." in name else ""
        for seg, _ in mod.segments:
            if mod.flat_name:
                yield (f"{parent}.{seg}" if parent else seg), mod, seg
            else:
                yield name, mod, seg


def lora_pairs_from_model(model: nn.Module, dtype=None):
    """Current LoRA weights of ``model`` as {module: {"A", "B"}} (one entry per adapted segment)."""
    pairs = {}
    for mname, lin, seg in _segment_module_names(model):
        if not lin.lora_rank or seg not in lin.lora_segments:
            continue
        r = lin.lora_rank
        j = lin.lora_segments.index(seg)
        sl = dict(lin.seg_slices())[seg]
        A = lin.lora_A.detach()[j * r:(j + 1) * r]
        B = lin.lora_B.detach()[sl, j * r:(j + 1) * r]
        pairs[mname] = {"A": A.to(dtype or A.dtype).cpu(), "B": B.to(dtype or B.dtype).cpu()}
    return pairs


@torch.no_grad()
def attach_lora(model: nn.Module, pairs, rank, alpha, strict=True):
    """Enable rank-``rank`` adapters exactly on the modules in ``pairs`` and load their weights."""
    by_lin: dict = {}
    names = {}
    for mname, lin, seg in _segment_module_names(model):
        names[mname] = (lin, seg)
    missing = [m for m in pairs if m not in names]
    if missing and strict:
        raise KeyError(f"LoRA modules not in the model: {missing[:5]}")
    for m in pairs:
        if m in names:
            lin, seg = names[m]
            by_lin.setdefault(id(lin), (lin, []))[1].append(seg)
    for lin, segs in by_lin.values():
        order = [s for s, _ in lin.segments if s in segs]
        lin.enable_lora(rank, alpha, segments=order)
    loaded = 0
    for m, p in pairs.items():
        if m not in names:
            continue
        lin, seg = names[m]
        r = lin.lora_rank
        j = lin.lora_segments.index(seg)
        sl = dict(lin.seg_slices())[seg]
        lin.lora_A[j * r:(j + 1) * r].copy_(p["A"].to(lin.lora_A.dtype))
        lin.lora_B[sl, j * r:(j + 1) * r].copy_(p["B"].to(lin.lora_B.dtype))
        loaded += 1
    if loaded != len(pairs) and strict:
        raise RuntimeError(f"loaded {loaded} of {len(pairs)} LoRA pairs")
    return loaded


@torch.no_grad()
def merge_lora(model: nn.Module):
    """Fold every adapter into its base weight (W += (alpha/r) B A) and drop the adapters."""
    for lin in [m for m in model.modules() if isinstance(m, SegLinear) and m.lora_rank]:
        lin.weight.add_(lin.lora_delta_weight().to(lin.weight.dtype))
        del lin.lora_A, lin.lora_B
        lin.lora_rank = 0
