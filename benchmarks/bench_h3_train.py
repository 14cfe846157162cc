"""H3 DMAD training iteration at the 33B shape (random-init weights), one sample per GPU, block weights
sharded over the ranks.

    torchrun --nproc-per-node 8 -m benchmarks.bench_h3_train [--critic lora|full] [--iters 1] [--warmup 1]

One iteration = one student stage (a rollout of 1..4 student evaluations, the last with grad, the critic
forward and backward through the frozen critic) and one critic stage (a no-grad rollout and three critic
forward / backward passes), as ``H3DMAD.train_iteration`` runs them; 124 frames at 1344x768 plus stereo
audio (37,966 tokens).  The rollout length is drawn per iteration (broadcast from rank 0), so iterations
differ in cost: the JSON line gives every iteration and their mean.  Device-timed (CUDA events), max over
ranks.  The reference publishes 6.7 h per 100 iterations with a LoRA critic and 5.5 h with a full critic
on 8 x H200 (train/h3/README.md:23-24): 241 s and 198 s per iteration.
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import time

import torch

HERE = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, HERE)


def main(argv=None):
    ap = argparse.ArgumentParser(description="H3 DMAD training iteration at the 33B shape")
    ap.add_argument("--critic", default="lora", choices=["lora", "full"])
    ap.add_argument("--iters", type=int, default=2)
    ap.add_argument("--warmup", type=int, default=1)
    ap.add_argument("--layers", type=int, default=None, help="debug only: fewer blocks (invalid for the headline)")
    a = ap.parse_args(argv)
    from dmad_b200.distill.h3_dmad import H3DMAD, H3DMADConfig
    from dmad_b200.models.h3 import H3Config
    from dmad_b200.parallel.dist import init_distributed

    rank, world, device = init_distributed(timeout_s=900)
    model = H3Config() if a.layers is None else H3Config(num_layers=a.layers)
    cfg = H3DMADConfig(model=model, fake_train_type=a.critic, shard_weights=world > 1)
    t0 = time.time()
    m = H3DMAD(cfg, device, dtype=torch.bfloat16, seed=0)
    with torch.no_grad():  # the output projections start at zero; random weights so gradients flow
        for net in (m.student, m.fake):
            for lin in (net.proj_out, net.audio_proj_out):
                lin.weight.normal_(0.0, 0.02, generator=torch.Generator(device=lin.weight.device).manual_seed(3))
    torch.cuda.synchronize()
    build_s = time.time() - t0
    for _ in range(a.warmup):
        m.train_iteration()
    torch.cuda.synchronize()
    torch.cuda.reset_peak_memory_stats()
    times = []
    for _ in range(a.iters):
        if world > 1:
            torch.distributed.barrier()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        m.train_iteration()
        e.record()
        e.synchronize()
        times.append(s.elapsed_time(e) / 1000.0)
    t = torch.tensor(times + [torch.cuda.max_memory_allocated() / 2 ** 30], device=device, dtype=torch.float64)
    if world > 1:
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    from dmad_b200.ops import check_device_status
    check_device_status()
    if rank == 0:
        its = [float(x) for x in t[:-1]]
        print(json.dumps({"metric": "H3 DMAD training: s per iteration (device-timed, max over ranks)",
                          "critic": a.critic, "gpus": world, "iterations_s": its, "mean_s": sum(its) / len(its),
                          "peak_gib": round(float(t[-1]), 1), "build_s": round(build_s, 1),
                          "config": {"model": f"H3-shaped DiT, {model.num_layers} blocks, hidden {model.dim}",
                                     "tokens_per_sample": 37966, "student_lora_rank": cfg.student_lora_rank,
                                     "weights": "random init", "dtype": "bf16",
                                     "sharding": "block weights sharded over the ranks" if world > 1 else "none"},
                          "reference_published_s_per_iteration_8xH200": {"lora": 241.2, "full": 198.0}[a.critic]}),
              flush=True)
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
