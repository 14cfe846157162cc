"""one fp32 CPU DMAD step (generator update + two-head critic update) of the
config-1 EDM U-Net (64x64x3, base channels 64, mult [1, 2, 2], one block per level, attention at
16x16, 1000 classes), batch 4, images U[-1, 1], labels U{0..999}, seed 0.

    python -m benchmarks.bench_edm_cpu [--steps 5] [--warmup 2] [--impl both|dmad_b200|reference]

Two arms on the same host, same shapes and the same step structure (train/image/main/edm/train_edm.py:
155-197: generator turn, clip, AdamW, EMA update, critic turn on the same generated batch, clip, AdamW):
* ``dmad_b200``: ``distill.edm_dmad.EDMDMAD.train_step``;
* ``reference``: the reference's own ``EDMUniModel`` (edm_unified_model.py), ``EDMGuidance``
  (edm_guidance.py), ``EDMPrecond`` / ``DhariwalUNet`` (third_party/edm/training/networks.py) and ``EMA``
  (main/utils.py), imported unmodified from the install under baseline/_ref/image (or the reference
  checkout).  The harness supplies what the reference gets from files and from its training script:
  random-init weights of the config-1 shape instead of the teacher pickle (``load_teacher_unet``), the
  critic heads sized for the config-1 bottleneck (the reference's ``make_binary_head`` is written for
  ImageNet's [768, 8, 8]; the harness builds the same conv / GroupNorm / SiLU stack for [128, 16, 16]),
  and the optimiser / EMA calls of ``train_one_step`` (its module imports wandb / accelerate / diffusers,
  which are not installed).
Both arms draw the critic's noise on the 1000-level Karras grid (the reference's stock path).  Prints one
JSON line per arm with the median wall time of a step (CPU: wall clock is the device clock).
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import sys
import time
import types

import torch
import torch.nn as nn

HERE = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, HERE)

B, RES, LABELS = 4, 64, 1000


def _reference_image_tree():
    cand = [os.path.join(HERE, "baseline", "_ref", "image")]
    try:
        ref = json.load(open(os.path.join(HERE, "BASELINE.json"))).get("reference_path")
        if ref:
            cand.append(os.path.join(ref, "train", "image"))
    except (OSError, ValueError):
        pass
    for c in cand:
        if os.path.isdir(os.path.join(c, "third_party", "edm")):
            return c
    return None


def _inputs(seed=0):
    g = torch.Generator().manual_seed(seed)
    eye = torch.eye(LABELS)
    real = torch.rand(B, 3, RES, RES, generator=g) * 2 - 1
    teach = torch.rand(B, 3, RES, RES, generator=g) * 2 - 1
    lr, lt, lab = (torch.randint(0, LABELS, (B,), generator=g) for _ in range(3))
    noise = torch.randn(B, 3, RES, RES, generator=g) * 80.0
    return {"real_image": real, "real_label": eye[lr], "second_real_image": teach, "second_real_label": eye[lt],
            "noise": noise, "labels": eye[lab]}


def _time(step, steps, warmup):
    for _ in range(warmup):
        step()
    ts = []
    for _ in range(steps):
        t0 = time.perf_counter()
        step()
        ts.append(time.perf_counter() - t0)
    return statistics.median(ts), ts


def run_ours(steps, warmup):
    from dmad_b200.distill.edm_dmad import EDMDMAD, EDMDMADConfig

    torch.manual_seed(0)
    # the settings the reference arm below is built with (its train_edm.py argument defaults where the
    # harness passes none): no generator spectral norm, uncapped critic noise, one EMA
    m = EDMDMAD(EDMDMADConfig(batch_size=B, critic_sigma="karras", generator_spectral_norm=False,
                              critic_max_timestep=None, gap_tau=2.0, r1_batch_size=2, ema_kimg=(0.5,), warmup_steps=0,
                              teacher_loss_weight=1.0, real_loss_weight=1.0), device="cpu")
    batch = _inputs()
    return _time(lambda: m.train_step(batch), steps, warmup)


def run_reference(steps, warmup):
    tree = _reference_image_tree()
    if tree is None:
        return None
    for p in (tree, os.path.join(tree, "third_party", "edm")):
        if p not in sys.path:
            sys.path.insert(0, p)
    from main.edm import edm_guidance, edm_unified_model
    from main.utils import EMA
    from third_party.edm.training.networks import EDMPrecond

    def config1_teacher(args):  # random init of the config-1 shape (stands in for the teacher pickle)
        unet = EDMPrecond(img_resolution=RES, img_channels=3, label_dim=LABELS, use_fp16=False, sigma_min=0,
                          sigma_max=float("inf"), sigma_data=0.5, model_type="DhariwalUNet", augment_dim=0,
                          model_channels=64, channel_mult=[1, 2, 2], channel_mult_emb=4, num_blocks=1,
                          attn_resolutions=[16], dropout=0.0, label_dropout=0)
        del unet.model.map_augment
        unet.model.map_augment = None
        return unet

    def config1_head():  # the reference head's layer stack, sized for the [128, 16, 16] bottleneck
        c = 128
        return nn.Sequential(nn.Conv2d(c, c, 4, 2, 1), nn.GroupNorm(32, c), nn.SiLU(),
                             nn.Conv2d(c, c, 4, 2, 1), nn.GroupNorm(32, c), nn.SiLU(),
                             nn.Conv2d(c, c, 4, 4, 0), nn.GroupNorm(32, c), nn.SiLU(), nn.Conv2d(c, 1, 1))

    edm_unified_model.load_teacher_unet = config1_teacher
    edm_guidance.make_binary_head = config1_head
    args = types.SimpleNamespace(
        pretrained_critic="", label_dim=LABELS, critic_freeze_backbone=False, critic_clean=False, r1_gamma=0.0,
        r1_batch_size=2, critic_max_timestep=None, teacher_gap_route=True, gap_tau=2.0, num_train_timesteps=1000,
        sigma_max=80.0, sigma_min=0.002, rho=7.0, min_step_percent=0.02, max_step_percent=0.98,
        critic_spectral_norm=True, generator_spectral_norm=False, dataset_name="imagenet", resolution=RES,
        use_fp16=False, sigma_data=0.5, model_id=None)
    torch.manual_seed(0)
    model = edm_unified_model.EDMUniModel(args, accelerator=None)
    opt_c = torch.optim.AdamW([p for p in model.guidance_model.parameters() if p.requires_grad], lr=2e-6,
                              betas=(0.0, 0.99))
    opt_g = torch.optim.AdamW(model.feedforward_model.parameters(), lr=2e-6, betas=(0.0, 0.99))
    ema = EMA(model.feedforward_model, decay=0.999)
    x = _inputs()
    real = {k: x[k] for k in ("real_image", "real_label", "second_real_image", "second_real_label")}
    sigma = torch.ones(B) * 80.0
    nstep = [0]

    def step():  # train_edm.py:155-197, minus logging
        model.train()
        gl, glog = model(x["noise"], sigma, x["labels"], real_train_dict=real, compute_generator_gradient=True,
                         generator_turn=True, guidance_turn=False)
        (gl["gen_teacher_loss"] + gl["gen_real_loss"]).backward()
        torch.nn.utils.clip_grad_norm_(model.feedforward_model.parameters(), 10.0)
        opt_g.step()
        opt_g.zero_grad()
        opt_c.zero_grad()
        nimg = (nstep[0] + 1) * B
        ema.decay = 0.5 ** (B / max(min(500.0, nimg * 0.05), 1e-8))
        ema.update(model.feedforward_model)
        cl, _ = model(x["noise"], sigma, x["labels"], real_train_dict=real, compute_generator_gradient=False,
                      generator_turn=False, guidance_turn=True, guidance_data_dict=glog["guidance_data_dict"])
        cl["critic_loss"].backward()
        torch.nn.utils.clip_grad_norm_(model.guidance_model.parameters(), 10.0)
        opt_c.step()
        opt_c.zero_grad()
        opt_g.zero_grad()
        nstep[0] += 1

    return _time(step, steps, warmup)


def main(argv=None):
    ap = argparse.ArgumentParser(description="config-1 CPU DMAD step")
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=2)
    ap.add_argument("--impl", default="both", choices=["both", "dmad_b200", "reference"])
    a = ap.parse_args(argv)
    cfg = {"model": "EDM U-Net 64x64x3, ch 64, mult [1,2,2], 1 block/level, attn 16x16, 1000 classes (config 1)",
           "batch": B, "dtype": "fp32", "device": "cpu", "threads": torch.get_num_threads()}
    if a.impl in ("both", "dmad_b200"):
        med, ts = run_ours(a.steps, a.warmup)
        print(json.dumps({"impl": "dmad_b200", "metric": "s per DMAD step (generator + critic update)",
                          "value": med, "unit": "s", "steps": ts, "config": cfg}))
    if a.impl in ("both", "reference"):
        r = run_reference(a.steps, a.warmup)
        if r is None:
            print(json.dumps({"impl": "reference", "unavailable": "reference image stack not found"}))
        else:
            print(json.dumps({"impl": "reference", "metric": "s per DMAD step (generator + critic update)",
                              "value": r[0], "unit": "s", "steps": r[1], "config": cfg}))


if __name__ == "__main__":
    main()
