"""Import a reference Wan DMAD / rCM training checkpoint (torch DCP) into this package's modules.

    python -m dmad_b200.tools.import_reference_checkpoint <run>/checkpoints/iter_000017000/model out.pt \\
        [--prefix net_ema.] [--release release.pth]

Parity: the reference's DCP layout (train/wan/rcm/checkpointers/dcp.py:486-612: one ``model`` directory
whose keys carry the distillation model's sub-module prefixes ``net.``, ``net_ema.``, ``net_fake_score.``
...) and its spectral-norm storage (torch parametrizations: ``<layer>.parametrizations.weight.original``,
``.0._u`` / ``.0._v`` of the power iteration and ``.1.gain`` of the frozen gain,
train/wan/scripts/dcp_to_pth_dmad.py:17-52).  The directory is read with torch's public DCP converter,
the sub-module of ``prefix`` is taken and its spectral-norm entries are renamed to this package's
``<layer>.weight`` / ``sn_u`` / ``sn_gain``; ``--release`` additionally folds the spectral norm and writes
the bf16 ``net.*`` file the samplers read (one power iteration from the stored u, as the reference's
converter does).
"""
from __future__ import annotations

import argparse
import os
import tempfile

import torch

MARK = ".parametrizations.weight."


def read_dcp(path: str) -> dict:
    """Every tensor of a DCP checkpoint directory, read in this process (no process group)."""
    from torch.distributed.checkpoint.format_utils import dcp_to_torch_save

    with tempfile.TemporaryDirectory() as d:
        out = os.path.join(d, "sd.pt")
        dcp_to_torch_save(path, out)
        return torch.load(out, map_location="cpu", weights_only=False)


def to_package_keys(sd: dict, prefix: str = "net_ema.") -> dict:
    """The ``prefix`` sub-module with spectral-norm parametrization keys renamed to this package's."""
    out = {}
    for k, v in sd.items():
        if not k.startswith(prefix):
            continue
        k = k[len(prefix):]
        if MARK in k:
            mod, rest = k.split(MARK)
            name = {"original": "weight", "0._u": "sn_u", "0._v": "sn_v", "1.gain": "sn_gain"}.get(rest)
            if name is None:
                continue
            k = f"{mod}.{name}"
        out[k] = v
    return out


def read_pretrained(path: str) -> dict:
    """A network state dict from a DCP checkpoint directory (the ``net_ema.`` sub-module when present,
    else ``net.``), a ``.safetensors`` file, or a torch file (a release ``net.*`` file or a plain state
    dict), with spectral-norm parametrization keys renamed to this package's."""
    if os.path.isdir(path):
        sd = read_dcp(path)
        prefix = "net_ema." if any(k.startswith("net_ema.") for k in sd) else "net."
        return to_package_keys(sd, prefix)
    if path.endswith(".safetensors"):
        from safetensors.torch import load_file
        sd = load_file(path)
    else:
        sd = torch.load(path, map_location="cpu", weights_only=False)
        for key in ("model", "state_dict", "module"):
            if isinstance(sd, dict) and isinstance(sd.get(key), dict):
                sd = sd[key]
    prefix = "net." if sd and all(k.startswith("net.") for k in sd) else ""
    return to_package_keys(sd, prefix)


def fold_spectral_norm(sd: dict) -> dict:
    """Plain weights: W g / sigma for every layer with ``sn_u`` / ``sn_gain`` (sigma after one power iteration
    from the stored u), other entries unchanged."""
    out = {}
    layers = {k[: -len(".sn_u")] for k in sd if k.endswith(".sn_u")}
    for k, v in sd.items():
        if k.endswith((".sn_u", ".sn_v", ".sn_gain")):
            continue
        mod = k[: -len(".weight")] if k.endswith(".weight") else None
        if mod in layers:
            W = v.float()
            u = sd[f"{mod}.sn_u"].float().reshape(-1)
            g = sd[f"{mod}.sn_gain"].float().reshape(())
            vv = torch.nn.functional.normalize(W.t() @ u, dim=0)
            uu = torch.nn.functional.normalize(W @ vv, dim=0)
            sigma = torch.dot(uu, W @ vv).clamp(min=1e-12)
            out[k] = g * W / sigma
        else:
            out[k] = v
    return out


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("dcp_dir")
    ap.add_argument("out", help="state dict for this package's WanModel (keys without the prefix)")
    ap.add_argument("--prefix", default="net_ema.", help="net_ema. (EMA student), net. (live) or net_fake_score.")
    ap.add_argument("--release", default=None, help="also write the SN-folded bf16 net.* release file")
    a = ap.parse_args(argv)
    sd = to_package_keys(read_dcp(a.dcp_dir), a.prefix)
    if not sd:
        raise SystemExit(f"no keys under {a.prefix!r} in {a.dcp_dir}")
    torch.save(sd, a.out)
    print(f"{len(sd)} tensors under {a.prefix} -> {a.out}")
    if a.release:
        rel = {f"net.{k}": (v.to(torch.bfloat16) if v.is_floating_point() else v)
               for k, v in fold_spectral_norm(sd).items()}
        torch.save(rel, a.release)
        print(f"release file -> {a.release}")


if __name__ == "__main__":
    main()
