"""Checkpoint-folder FID evaluator of EDM DMAD runs, next to the training job.

Counterpart of the reference's ``train/image/main/edm/test_folder_edm.py`` (protocol :1-12, sampling
:96-124, statistics :127-143, EMA files :153-166): it watches a training output folder and evaluates every
newly published checkpoint's generator EMAs (``pytorch_model_ema.bin`` -> ``fid``,
``pytorch_model_ema_<K>.bin`` -> ``fid_ema_<K>``, the files the EDM trainer exports): N one-step samples
(noise * sigma at sigma = ``--conditioning-sigma``, class labels cycling over the classes, one fixed seed),
images quantised as ``clamp((x + 1) * 127.5, 0, 255)`` to uint8, the caller's Inception detector, FID
against reference statistics.  Results accumulate in ``<folder>/stats.json`` (one entry per checkpoint; the
reference also logs them to wandb).  One difference: the reference starts its covariance sum from ones; here
it starts from zeros, as its ``fid.py`` does (the ones add 1 / (N - 1) to every covariance entry).

    python -m dmad_b200.tools.edm_eval_folder --folder outputs/edm_dmad --ref imagenet-64x64.npz \\
        --detector inception-2015-12-05.pt [--run-once]
"""
from __future__ import annotations

import argparse
import glob
import json
import os
import re
import time

import numpy as np
import torch

from ..models.edm import config1_unet
from ..runtime.checkpoint import completed_checkpoints, parse_checkpoint_iteration
from ..samplers.edm import frechet_distance
from .edm_fid import batch_stats, load_detector


def ema_weight_files(checkpoint: str) -> list[tuple[str, str]]:
    """[(metric name, path)]: the primary EMA, then the extra ones by half-life."""
    out = []
    primary = os.path.join(checkpoint, "pytorch_model_ema.bin")
    if os.path.isfile(primary):
        out.append(("fid", primary))
    extra = []
    for path in glob.glob(os.path.join(checkpoint, "pytorch_model_ema_*.bin")):
        m = re.fullmatch(r"pytorch_model_ema_(\d+)\.bin", os.path.basename(path))
        if m:
            extra.append((int(m.group(1)), path))
    return out + [(f"fid_ema_{k}", p) for k, p in sorted(extra)]


@torch.no_grad()
def one_step_samples(net, num: int, batch: int, seed: int, label_dim: int, resolution: int, sigma: float, device):
    """uint8 NCHW batches of the generator's one-step samples (labels i mod label_dim, one seed)."""
    torch.manual_seed(seed)
    labels = torch.arange(0, num + batch, device=device) % label_dim
    eye = torch.eye(label_dim, device=device)
    done = 0
    while done < num:
        n = min(batch, num - done)
        noise = torch.randn(batch, 3, resolution, resolution, device=device)
        x = net(noise * sigma, torch.full((batch,), sigma, device=device), eye[labels[done:done + batch]])
        yield ((x[:n] + 1.0) * 127.5).clamp(0, 255).to(torch.uint8).cpu()
        done += n


def evaluate_checkpoint(ckpt: str, detector, ref: dict, args) -> dict:
    res = {"iteration": parse_checkpoint_iteration(ckpt)}
    for metric, path in ema_weight_files(ckpt):
        net = config1_unet(args.label_dim).to(args.device).eval()
        net.load_state_dict(torch.load(path, map_location=args.device))
        batches = one_step_samples(net, args.num, args.batch, args.seed, args.label_dim, args.resolution,
                                   args.conditioning_sigma, args.device)
        mu, sigma = batch_stats(batches, detector, args.device)
        res[metric] = frechet_distance(mu, sigma, ref["mu"], ref["sigma"])
    return res


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--folder", required=True, help="training output folder receiving checkpoint-* folders")
    ap.add_argument("--ref", required=True, help="reference FID statistics (.npz with mu / sigma)")
    ap.add_argument("--detector", required=True, help="Inception-v3 feature network (TorchScript, or the "
                                                     "reference's pickle with --trust-pickle)")
    ap.add_argument("--trust-pickle", action="store_true")
    ap.add_argument("--num", type=int, default=50000, help="samples per EMA")
    ap.add_argument("--batch", type=int, default=128)
    ap.add_argument("--seed", type=int, default=10)
    ap.add_argument("--label-dim", type=int, default=1000)
    ap.add_argument("--resolution", type=int, default=64)
    ap.add_argument("--conditioning-sigma", type=float, default=80.0)
    ap.add_argument("--run-once", action="store_true", help="evaluate what is in the folder now and exit")
    ap.add_argument("--poll-s", type=float, default=60.0)
    ap.add_argument("--device", default="cuda" if torch.cuda.is_available() else "cpu")
    a = ap.parse_args(argv)
    detector = load_detector(a.detector, a.device, a.trust_pickle)
    ref = dict(np.load(a.ref))
    stats_path = os.path.join(a.folder, "stats.json")
    stats = json.load(open(stats_path)) if os.path.isfile(stats_path) else {}
    while True:
        for ckpt in completed_checkpoints(a.folder):
            name = os.path.basename(ckpt)
            if name in stats or not ema_weight_files(ckpt):
                continue
            stats[name] = evaluate_checkpoint(ckpt, detector, ref, a)
            print(json.dumps({name: stats[name]}), flush=True)
            tmp = stats_path + ".tmp"
            with open(tmp, "w") as f:
                json.dump(stats, f, indent=1)
            os.replace(tmp, stats_path)
        if a.run_once:
            return stats
        time.sleep(a.poll_s)


if __name__ == "__main__":
    main()
