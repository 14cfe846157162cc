"""Convert an H3 DMAD student LoRA (Diffusers layout) to the ComfyUI MiniMax-H3 layout, exactly.

Parity: tools/convert_lora_comfyui.py:52-99 of the reference.  ComfyUI fuses q/k/v into one
``qkv_proj`` and orders the SwiGLU hidden layer ``[gate; value]``, while the Diffusers layout has
separate ``to_q/to_k/to_v`` and ``[value; gate]``.  The mapping (a file format, kept as it must be):

  transformer_blocks.N.attn.to_{q,k,v} -> diffusion_model.blocks.N.attn.qkv_proj
        A = [A_q; A_k; A_v] (3r x in), B = block_diag(B_q, B_k, B_v) (3 out x 3r), alpha = 3r
  transformer_blocks.N.attn.to_out.0   -> diffusion_model.blocks.N.attn.out_proj
  transformer_blocks.N.ff.net.0.proj   -> diffusion_model.blocks.N.mlp.fc1   (B halves swapped)
  transformer_blocks.N.ff.net.2        -> diffusion_model.blocks.N.mlp.fc2
  token_refiner.refiner_blocks.N.*     -> diffusion_model.token_refiner.blocks.N.* (same four)

    python -m dmad_b200.tools.lora_comfyui in.safetensors out.safetensors
"""
from __future__ import annotations

import argparse
import os

import torch

from ..lora import lora_rank_alpha, read_lora_file

_TAILS = {"attn.to_out.0": "attn.out_proj", "ff.net.0.proj": "mlp.fc1", "ff.net.2": "mlp.fc2"}


def split_module(module: str):
    if module.startswith("transformer_blocks."):
        _, n, tail = module.split(".", 2)
        return f"diffusion_model.blocks.{n}", tail
    if module.startswith("token_refiner.refiner_blocks."):
        _, _, n, tail = module.split(".", 3)
        return f"diffusion_model.token_refiner.blocks.{n}", tail
    raise ValueError(f"unexpected LoRA module {module}")


def _swap_halves(b):
    h = b.shape[0] // 2
    return torch.cat([b[h:], b[:h]], dim=0)


def convert(pairs, rank, alpha):
    if float(alpha) != float(rank):
        raise ValueError(f"alpha {alpha} != rank {rank}; the ComfyUI alpha entries assume alpha = rank")
    grouped: dict = {}
    for module, p in pairs.items():
        prefix, tail = split_module(module)
        grouped.setdefault(prefix, {})[tail] = p
    out = {}
    for prefix, mods in sorted(grouped.items()):
        qkv = [mods.pop(f"attn.to_{c}") for c in "qkv"]
        A = torch.cat([p["A"] for p in qkv], dim=0)
        B = torch.block_diag(*[p["B"] for p in qkv]).to(qkv[0]["B"].dtype)
        out[f"{prefix}.attn.qkv_proj.lora_A.weight"] = A.contiguous()
        out[f"{prefix}.attn.qkv_proj.lora_B.weight"] = B.contiguous()
        out[f"{prefix}.attn.qkv_proj.alpha"] = torch.tensor(float(A.shape[0]), dtype=B.dtype)
        for tail, name in _TAILS.items():
            p = mods.pop(tail)
            B = _swap_halves(p["B"]) if name == "mlp.fc1" else p["B"]
            out[f"{prefix}.{name}.lora_A.weight"] = p["A"].contiguous()
            out[f"{prefix}.{name}.lora_B.weight"] = B.contiguous()
            out[f"{prefix}.{name}.alpha"] = torch.tensor(float(p["A"].shape[0]), dtype=B.dtype)
        if mods:
            raise ValueError(f"modules left unconverted under {prefix}: {sorted(mods)}")
    return out


def verify(pairs, out):
    """Every converted adapter reproduces the original update B A bit-exactly (fp32, CPU)."""
    for module, p in pairs.items():
        prefix, tail = split_module(module)
        want = p["B"].float() @ p["A"].float()
        if tail in ("attn.to_q", "attn.to_k", "attn.to_v"):
            i = "qkv".index(tail[-1])
            A = out[f"{prefix}.attn.qkv_proj.lora_A.weight"].float()
            B = out[f"{prefix}.attn.qkv_proj.lora_B.weight"].float()
            o = want.shape[0]
            got = B[i * o:(i + 1) * o] @ A
        else:
            name = _TAILS[tail]
            got = out[f"{prefix}.{name}.lora_B.weight"].float() @ out[f"{prefix}.{name}.lora_A.weight"].float()
            if name == "mlp.fc1":
                got = _swap_halves(got)
        if not torch.equal(got, want):
            raise AssertionError(f"{module}: converted update differs by {(got - want).abs().max():.3g}")


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("source")
    ap.add_argument("output")
    ap.add_argument("--no-verify", action="store_true")
    a = ap.parse_args(argv)
    from safetensors.torch import save_file

    pairs, meta = read_lora_file(a.source)
    rank, alpha = lora_rank_alpha(pairs, meta)
    out = convert(pairs, rank, alpha)
    if not a.no_verify:
        verify(pairs, out)
    md = {"format": "pt", "converted_layout": "comfyui_minimax_h3", "source": os.path.basename(a.source),
          "lora_rank": str(rank), "lora_alpha": str(alpha)}
    os.makedirs(os.path.dirname(os.path.abspath(a.output)) or ".", exist_ok=True)
    save_file(out, a.output, metadata=md)
    print(f"wrote {a.output}: {sum(k.endswith('.weight') for k in out)} tensors")


if __name__ == "__main__":
    main()
