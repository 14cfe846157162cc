"""Export an image generator (EDM or SDXL-shaped U-Net) with its spectral norms folded.

    python -m dmad_b200.tools.export_unet <checkpoint-dir> <out.pt> [--ema-kimg 0.5] [--dtype fp16]

Parity: train/image/main/sdxl/export_unet.py (SN-folded fp16 UNet state dict) and the FID path of
train/image/main/edm/test_folder_edm.py, which folds the SN of the EMA generator before sampling.
``fold_spectral_norm`` (``algorithms.spectral``) replaces every normalised weight by the effective
weight of the network in eval mode and turns the layer back into its plain class, so the plain
network class loads the result.
"""
from __future__ import annotations

import argparse
import copy

import torch
from ..algorithms.spectral import fold_spectral_norm


def plain_state_dict(module: torch.nn.Module, dtype=torch.float16) -> dict:
    m = copy.deepcopy(module).eval()
    fold_spectral_norm(m)
    return {k: (v.to(dtype) if v.is_floating_point() else v) for k, v in m.state_dict().items()}


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("checkpoint")
    ap.add_argument("out")
    ap.add_argument("--family", default="edm_dmad", choices=["edm_dmad", "sdxl_dmad"])
    ap.add_argument("--dtype", default="fp16", choices=["fp16", "bf16", "fp32"])
    a = ap.parse_args(argv)
    import os
    import yaml
    from ..train.registry import build_model

    cfg = yaml.safe_load(open(os.path.join(a.checkpoint, "config.yaml")))
    adapter = build_model(cfg, torch.device("cpu"))
    shared = torch.load(os.path.join(a.checkpoint, "shared.pt"), map_location="cpu", weights_only=False)
    adapter.load_state_dicts(shared, None)
    dt = {"fp16": torch.float16, "bf16": torch.bfloat16, "fp32": torch.float32}[a.dtype]
    sd = plain_state_dict(adapter.modules["generator"], dt)
    torch.save(sd, a.out)
    print(f"wrote {len(sd)} tensors to {a.out}")


if __name__ == "__main__":
    main()
