"""Training checkpoint -> release ``.pth`` (student EMA, spectral norm folded, bf16 ``net.*`` keys).

    python -m dmad_b200.tools.export_release <checkpoint-dir> <out.pth> [--no-ema] [--dtype bf16|fp16|fp32]

Parity: train/wan/scripts/dcp_to_pth_dmad.py:180-209 (take the EMA weights of the student, fold the
frozen-gain spectral norm with one power iteration from the stored u, save ``net.*`` in bf16).
The EMA lives as per-rank fp32 shards (``rank*.pt``) of the sharded optimiser; it is rebuilt
offline from the layout the checkpoint records, so no process group is needed.  Works on CPU.
"""
from __future__ import annotations

import argparse
import glob
import os

import torch
import yaml


def build_student(cfg: dict):
    from ..distill.wan_dmad import WanDMADConfig
    from ..models.wan import WanConfig, WanModel, wan_config
    from ..runtime.config import to_dataclass
    import math

    m = cfg.get("model", {})
    net = m.get("net", "wan2.1-1.3b")
    if isinstance(net, str):
        ncfg = wan_config(net)
    else:
        net = dict(net)
        base = net.pop("name", None)
        ncfg = wan_config(base, **net) if base else to_dataclass(WanConfig, net)
    d = to_dataclass(WanDMADConfig, m.get("distill") or {})
    model = WanModel(ncfg)
    if d.generator_spectral_norm:
        model.enable_spectral_norm(range(math.ceil(ncfg.num_layers * d.sn_generator_frac)), power_iters=1)
    if d.student_lora_rank:
        model.enable_lora(d.student_lora_rank)
    return model


def export(ckpt_dir: str, out_path: str, use_ema: bool = True, dtype=torch.bfloat16) -> dict:
    from ..models.layers import SegLinear
    from ..parallel.zero import tensors_from_shards

    with open(os.path.join(ckpt_dir, "config.yaml")) as f:
        cfg = yaml.safe_load(f)
    shared = torch.load(os.path.join(ckpt_dir, "shared.pt"), map_location="cpu", weights_only=False)
    model = build_student(cfg)
    model.load_state_dict(shared["net"])
    if use_ema:
        if "student_layout" in shared:
            ranks = [torch.load(p, map_location="cpu", weights_only=False)["opt_student"]
                     for p in sorted(glob.glob(os.path.join(ckpt_dir, "rank*.pt")))]
            ema = tensors_from_shards(shared["student_layout"], ranks, "ema")
        elif shared.get("ema") is not None:
            trainable = [n for n, p in model.named_parameters() if p.requires_grad]
            ema = dict(zip(trainable, shared["ema"]))
        else:
            raise RuntimeError("checkpoint has no EMA (trained with ema_enabled=false?); use --no-ema")
        params = dict(model.named_parameters())
        with torch.no_grad():
            for n, t in ema.items():
                params[n].copy_(t.to(params[n].dtype))
    # fold SN and LoRA into plain weights; drop the SN buffers
    with torch.no_grad():
        for mod in model.modules():
            if isinstance(mod, SegLinear):
                w = mod.folded_weight().float()
                if mod.lora_rank:
                    w = w + mod.lora_delta_weight().float()
                    mod.lora_rank = 0
                mod.weight.copy_(w.to(mod.weight.dtype))
                mod.sn_enabled = False
    sd = {}
    for k, v in model.state_dict().items():
        if k.endswith(("sn_u", "sn_v", "sn_gain", "sn_mask")) or ".lora_" in k:
            continue
        sd[f"net.{k}"] = v.to(dtype) if v.is_floating_point() else v
    tmp = out_path + ".tmp"
    torch.save(sd, tmp)
    os.replace(tmp, out_path)
    return sd


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("checkpoint")
    ap.add_argument("out")
    ap.add_argument("--no-ema", action="store_true")
    ap.add_argument("--dtype", default="bf16", choices=["bf16", "fp16", "fp32"])
    a = ap.parse_args(argv)
    dt = {"bf16": torch.bfloat16, "fp16": torch.float16, "fp32": torch.float32}[a.dtype]
    sd = export(a.checkpoint, a.out, use_ema=not a.no_ema, dtype=dt)
    print(f"wrote {len(sd)} tensors to {a.out}")


if __name__ == "__main__":
    main()
