"""SDXL-shaped U-Net (2.6B; channels 320/640/1280, transformer depths 0/2/10, cross-attention
dim 2048) 4-step DMAD training in bf16, data parallel, batch 4 per GPU, 4x128x128 latents, 77x2048 text and a
pooled 1280 vector, N(0,1) inputs, random-init weights.

    torchrun --nproc-per-node N -m benchmarks.bench_sdxl [--dp sharded|nccl] [--steps 3] [--warmup 2]

One step = ``SDXLDMAD.train_step`` (backward simulation, generator update, critic update on the same batch).
``--dp sharded``: the fused reduce-scatter / AdamW / all-gather kernel; ``--dp nccl``: NCCL all-reduce of the
gradients and torch's AdamW on every rank (the library path; the reference's SDXL trainer cannot be built
here: its diffusers dependency is missing, so this is the comparison).  Device-timed, max over ranks; prints
images/s for the whole job.
"""
from __future__ import annotations

import argparse
import json
import os
import sys

import torch

HERE = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, HERE)


def main(argv=None):
    ap = argparse.ArgumentParser(description="config-4 SDXL DMAD step")
    ap.add_argument("--dp", default="sharded", choices=["sharded", "nccl"])
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=2)
    ap.add_argument("--batch", type=int, default=4)
    a = ap.parse_args(argv)
    from dmad_b200.distill.sdxl_dmad import SDXLDMAD, SDXLDMADConfig
    from dmad_b200.parallel.dist import init_distributed

    rank, world, device = init_distributed(timeout_s=900)
    cfg = SDXLDMADConfig(batch_size=a.batch, dp_optimizer=a.dp)
    m = SDXLDMAD(cfg, device=device, dtype=torch.bfloat16, seed=0)
    g = torch.Generator().manual_seed(100 + rank)
    B, r = a.batch, cfg.latent
    batch = {"noise": torch.randn(B, 4, r, r, generator=g).to(device),
             "real": torch.randn(B, 4, r, r, generator=g).to(device),
             "teacher": torch.randn(B, 4, r, r, generator=g).to(device),
             "ctx": torch.randn(B, 77, 2048, generator=g).to(device, torch.bfloat16),
             "pooled": torch.randn(B, 1280, generator=g).to(device, torch.bfloat16)}
    for _ in range(a.warmup):
        m.train_step(batch)
    torch.cuda.synchronize()
    torch.cuda.reset_peak_memory_stats()
    times = []
    for _ in range(a.steps):
        if world > 1:
            torch.distributed.barrier()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        m.train_step(batch)
        e.record()
        e.synchronize()
        times.append(s.elapsed_time(e))
    ms = torch.tensor([sum(times) / len(times), torch.cuda.max_memory_allocated() / 2 ** 30], device=device,
                      dtype=torch.float64)
    if world > 1:
        torch.distributed.all_reduce(ms, op=torch.distributed.ReduceOp.MAX)
    if rank == 0:
        print(json.dumps({"metric": "SDXL DMAD training images/s (device-timed, max over ranks)", "dp": a.dp,
                          "gpus": world, "ms_per_step": float(ms[0]), "images_per_s": world * B / (float(ms[0]) / 1e3),
                          "peak_gib": round(float(ms[1]), 1),
                          "config": {"model": "SDXL-shaped U-Net 2.6B", "batch_per_gpu": B, "latents": "4x128x128",
                                     "text": "77x2048 + pooled 1280", "dtype": "bf16", "weights": "random init"}}),
              flush=True)
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
