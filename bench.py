"""Headline benchmark: DMAD training throughput (samples/s) and 4-step generation latency
(s/clip) of the Wan2.1-T2V-1.3B-shaped DiT, on 1..8 B200s of one node.

One benchmark step = one full DMAD cycle on one sample per GPU: a generator iteration
followed by a critic iteration (the reference alternates them 1:1, student_update_freq=2).
Both include backward simulation (1..4 student evaluations, cycling as in the reference),
the critic forwards, backward, and the AdamW updates (plus the EMA update of the student).

    python bench.py --gpus N --steps K --warmup W            # this framework
    python bench.py --impl reference --gpus N --steps K --warmup W   # the reference build

For N > 1 launch with torchrun (one rank per GPU, NCCL); throughput is the whole-job
aggregate and every timing is the max over ranks of CUDA-event device time.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)

LATENT_SHAPE = (16, 21, 60, 104)   # 81 frames at 480x832, VAE stride 4x8x8
TEXT_SHAPE = (512, 4096)           # umT5-shaped context
SEQ_LEN = 21 * 30 * 52             # tokens after 1x2x2 patchify
L2_BYTES = 126 * 1024 * 1024


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=4)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="dmad_b200", choices=["dmad_b200", "reference"])
    ap.add_argument("--model", default="wan2.1-1.3b")
    ap.add_argument("--layers", type=int, default=None, help="debug only: fewer blocks (invalid for the headline)")
    ap.add_argument("--frames", type=int, default=LATENT_SHAPE[1], help="debug only: latent frames")
    ap.add_argument("--gen-runs", type=int, default=2)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--count-launches", type=int, default=1)
    ap.add_argument("--profile", default=None, help="write a per-kernel time table of one cycle to this path")
    ap.add_argument("--cp", type=int, default=1, help="context-parallel group size (config 3: 8)")
    ap.add_argument("--cp-impl", default="fused", choices=["fused", "nccl", "ring", "hybrid"])
    ap.add_argument("--ulysses-size", type=int, default=None, help="hybrid CP: ranks per Ulysses group")
    ap.add_argument("--lora", type=int, default=0, help="LoRA rank of the student (config 3: 128)")
    ap.add_argument("--cm-loss-scale", type=float, default=None,
                    help="weight of the sCM consistency term (flash-attention JVP path); default 100 for the 14B "
                         "config (BASELINE config 3), 0 for the 1.3B DMAD config (the reference's DMAD recipe)")
    ap.add_argument("--dp-path", default="auto", choices=["auto", "nvls", "p2p"],
                    help="fused optimiser transport: NVLS multimem or P2P peer loads/stores (auto: P2P up to 2 "
                         "GPUs, NVLS above, as measured by benchmarks/bench_collectives.py)")
    ap.add_argument("--fsdp", action="store_true",
                    help="FSDP-style sharding of the trainable block weights (critic, and the student unless LoRA)")
    ap.add_argument("--fsdp-shard-size", type=int, default=None,
                    help="with --fsdp: shard within groups of this many ranks, replicate across them (HSDP)")
    ap.add_argument("--dp-optimizer", default="sharded", choices=["sharded", "replicated"],
                    help="sharded: fused reduce-scatter/AdamW/all-gather kernel; replicated: NCCL all-reduce baseline")
    return ap.parse_args()


class ClockSampler:
    """Samples nvidia-smi clocks / throttle reasons during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = None

    def start(self):
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in open(self.path):
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax = float(parts[2])
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        os.unlink(self.path)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax, "reasons": sorted(reasons),
                "samples": len(sm)}


def make_host_batch(frames: int, seed: int):
    g = torch.Generator().manual_seed(seed)
    shp = (1, LATENT_SHAPE[0], frames, LATENT_SHAPE[2], LATENT_SHAPE[3])
    b = {
        "latents": torch.randn(shp, generator=g),            # teacher samples (Q)
        "real_latents": torch.randn(shp, generator=g),       # caption-paired real latents (T)
        "context": torch.randn((1,) + TEXT_SHAPE, generator=g).to(torch.bfloat16),
    }
    return {k: v.pin_memory() for k, v in b.items()}


def to_device(host, device):
    return {k: v.to(device, non_blocking=True) for k, v in host.items()}


def flush_l2(buf):
    buf.add_(1)


def count_my_kernels(fn, prefixes=("dmad",)) -> int:
    """Number of kernels from this package launched by one call of fn (torch profiler, untimed)."""
    from torch.profiler import ProfilerActivity, profile

    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        fn()
        torch.cuda.synchronize()
    n = 0
    for evt in prof.events():
        if evt.device_type is not None and "CUDA" in str(evt.device_type) and any(p in evt.name for p in prefixes):
            n += 1
    return n


# ---------------------------------------------------------------------- process-group plumbing
# (plain torch.distributed, so the reference arm imports nothing of this package)


def init_distributed(timeout_s: float):
    import datetime

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    if world > 1 and not torch.distributed.is_initialized():
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=timeout_s), device_id=device)
    return rank, world, device


def barrier():
    if torch.distributed.is_initialized():
        torch.distributed.barrier()


def max_over_ranks(x: float) -> float:
    if not torch.distributed.is_initialized():
        return float(x)
    t = torch.tensor([float(x)], dtype=torch.float64, device="cuda")
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return float(t.item())


def _dp_desc(trainer, args):
    if args.impl == "reference":
        return "reference: NCCL gradient all-reduce + master-weight AdamW"
    opt = getattr(trainer, "opt_student", None)
    if getattr(trainer, "fsdp", None):
        return ("FSDP-sharded block weights: peer-memory gather one block ahead, per-block reduce-scatter kernel "
                "in backward, AdamW on the shards; other weights: fused reduce-scatter+AdamW+all-gather")
    if args.dp_optimizer == "sharded" and opt is not None and hasattr(opt, "multicast"):
        return "sharded fp32 state; fused reduce-scatter+AdamW+all-gather kernel (" + \
            ("NVLS multimem" if opt.multicast else "P2P peer loads/stores") + ")"
    return "replicated: NCCL all-reduce + multi-tensor AdamW"


def main():
    args = parse()
    rank, world, device = init_distributed(timeout_s=900)
    assert world == args.gpus, f"--gpus {args.gpus} but WORLD_SIZE {world}"
    torch.backends.cuda.matmul.allow_tf32 = True
    torch.backends.cudnn.allow_tf32 = True
    headline_ok = args.layers is None and args.frames == LATENT_SHAPE[1]

    if args.impl == "reference":
        from baseline.reference_arm import build_reference_trainer
        trainer = build_reference_trainer(args, device)
        if trainer is None:
            return
    else:
        from dmad_b200.distill.wan_dmad import WanDMAD, WanDMADConfig
        from dmad_b200.models.wan import wan_config

        over = {"num_layers": args.layers} if args.layers else {}
        multicast = {"nvls": True, "p2p": False, "auto": world > 2}[args.dp_path]
        cfg = WanDMADConfig(net=wan_config(args.model, **over), dp_optimizer=args.dp_optimizer, dp_multicast=multicast,
                            fsdp_trainable=args.fsdp, fsdp_shard_size=args.fsdp_shard_size)
        cfg.checkpoint_critic_blocks_student_phase = cfg.net.num_layers
        big = "14b" in args.model.lower()
        cfg.loss_scale = args.cm_loss_scale if args.cm_loss_scale is not None else (100.0 if big else 0.0)
        if big:  # the reference's 14B DMAD experiment: critic checkpointed block-wise, lr 1e-6
            cfg.checkpoint_critic_blocks = cfg.net.num_layers
            cfg.lr = cfg.critic_lr = 1e-6
        if args.lora:
            cfg.student_lora_rank = args.lora
            cfg.shard_frozen = world > 1
            cfg.checkpoint_student_blocks = cfg.net.num_layers
        trainer = WanDMAD(cfg, device=device, dtype=torch.bfloat16, seed=0)
        if args.cp > 1:
            from dmad_b200.parallel.cp import make_context_parallel
            from dmad_b200.train.trainer import make_cp_group
            cpc = make_context_parallel(make_cp_group(args.cp), impl=args.cp_impl, device=device,
                                        ulysses_size=args.ulysses_size)
            for net in trainer.context_parallel_nets():
                net.enable_context_parallel(cpc)

    host = make_host_batch(args.frames, seed=1234 + rank // max(1, args.cp))
    batch = to_device(host, device)
    l2buf = torch.empty(2 * L2_BYTES // 4, dtype=torch.float32, device=device)
    it = [0]

    def cycle(b):
        o1 = trainer.training_step(b, it[0])
        o2 = trainer.training_step(b, it[0] + 1)
        it[0] += 2
        return o1, o2

    def mem(phase):
        """Peak device memory of the phase just finished (stderr), then a fresh peak for the next one."""
        if torch.cuda.is_available() and rank == 0:
            print(f"# memory after {phase}: peak {torch.cuda.max_memory_allocated() / 2**30:.1f} GiB, "
                  f"now {torch.cuda.memory_allocated() / 2**30:.1f} GiB", file=sys.stderr, flush=True)
        if torch.cuda.is_available():
            torch.cuda.reset_peak_memory_stats()

    def optional(phase, fn):
        """Runs an optional phase; its failure nulls its own field, not the timed result."""
        try:
            return fn()
        except Exception as e:  # noqa: BLE001 - reported, then the line is printed without this field
            if rank == 0:
                print(f"# {phase} failed: {e!r}", file=sys.stderr, flush=True)
            torch.cuda.empty_cache()
            return None
        finally:
            mem(phase)

    mem("setup")
    # ------------------------------------------------------------------ warm-up
    for _ in range(args.warmup):
        cycle(batch)
    torch.cuda.synchronize()
    barrier()
    mem("warm-up")

    # ------------------------------------------------------------------ device-timed loop
    clocks = ClockSampler(torch.cuda.current_device())
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    per_step = []
    barrier()
    torch.cuda.synchronize()
    clocks.start()
    for _ in range(args.steps):
        flush_l2(l2buf)
        start.record()
        cycle(batch)
        end.record()
        end.synchronize()
        per_step.append(start.elapsed_time(end))
    torch.cuda.synchronize()
    barrier()
    clk = clocks.stop()
    dev_ms = max_over_ranks(sum(per_step) / len(per_step))
    mem("timed loop")

    # ------------------------------------------------------------------ end-to-end loop (public API,
    # pinned H2D of the step's inputs and D2H of the step's losses inside the timed region)
    def run_e2e():
        h2d = sum(v.numel() * v.element_size() for v in host.values())
        loss_host = torch.empty(2, dtype=torch.float32).pin_memory()
        barrier()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        s_ev, e_ev = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s_ev.record()
        for _ in range(args.steps):
            b = to_device(host, device)
            o1, o2 = cycle(b)
            ls = torch.stack([torch.as_tensor(o1.get("dmad_g_loss", 0.0), device=device).float().reshape(()),
                              torch.as_tensor(o2.get("dmad_d_loss", 0.0), device=device).float().reshape(())])
            loss_host.copy_(ls, non_blocking=True)
            torch.cuda.current_stream().synchronize()
        e_ev.record()
        e_ev.synchronize()
        wall = (time.perf_counter() - t0) * 1000 / args.steps
        e2e_ms = max_over_ranks(max(wall, s_ev.elapsed_time(e_ev) / args.steps))
        return {"value": (world // args.cp) / (e2e_ms / 1000.0), "unit": "samples/s", "h2d_bytes_per_step": int(h2d),
                "d2h_bytes_per_step": int(loss_host.numel() * 4), "ms_per_step": e2e_ms}

    e2e = None if args.no_e2e else optional("e2e loop", run_e2e)

    # ------------------------------------------------------------------ 4-step generation latency
    def run_gen():
        ctx = batch["context"]
        shp = (1,) + (LATENT_SHAPE[0], args.frames, LATENT_SHAPE[2], LATENT_SHAPE[3])
        trainer.generate(ctx, shp, num_steps=4)
        times = []
        for _ in range(args.gen_runs):
            barrier()
            s2, e2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s2.record()
            trainer.generate(ctx, shp, num_steps=4)
            e2.record()
            e2.synchronize()
            times.append(s2.elapsed_time(e2) / 1000.0)
        return max_over_ranks(min(times))

    gen_s = optional("4-step generation", run_gen) if args.gen_runs > 0 else None

    if args.profile and rank == 0:
        from torch.profiler import ProfilerActivity, profile

        with profile(activities=[ProfilerActivity.CUDA, ProfilerActivity.CPU]) as prof:
            cycle(batch)
            torch.cuda.synchronize()
        with open(args.profile, "w") as f:
            f.write(prof.key_averages().table(sort_by="cuda_time_total", row_limit=60, max_name_column_width=90))

    launches = None
    if args.count_launches and args.impl == "dmad_b200":
        per_cycle = optional("launch count", lambda: count_my_kernels(lambda: cycle(batch)))
        launches = None if per_cycle is None else per_cycle * args.steps

    if args.impl == "dmad_b200":
        from dmad_b200 import ops
        try:
            ops.check_device_status()
        except Exception as e:
            if rank == 0:
                print(f"# device status: {e}", file=sys.stderr)
            raise

    value = (world // args.cp) / (dev_ms / 1000.0)
    out = {
        # the metric named by BASELINE.json; "value" is the training throughput, the 4-step generation
        # latency is "gen_latency_s_per_clip"
        "metric": "DMAD train samples/s and 4-step video gen latency (s/clip), device-timed max over ranks, "
                  "1/2/4/8 B200",
        "value": value,
        "unit": "samples/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": dev_ms,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic N(0,1) latents/context, random-init weights",
        "config": {"model": (f"{args.model}-shaped DiT (BASELINE config {'3' if '14b' in args.model else '2'})"
                             if headline_ok else "DEBUG (invalid)"),
                   "global_batch": world // args.cp, "seq_len": SEQ_LEN if headline_ok else None,
                   "latents": f"16x{args.frames}x60x104", "text": "512x4096",
                   "parallelism": f"dp{world // args.cp}" + (f"-cp{args.cp}-{args.cp_impl}" if args.cp > 1 else ""),
                   "student_lora_rank": args.lora or None,
                   "scm_loss_scale": (None if args.impl == "reference" else trainer.cfg.loss_scale),
                   "step": "1 generator + 1 critic DMAD iteration",
                   "dp_optimizer": _dp_desc(trainer, args),
                   "l2": "flushed (write of a 252 MB buffer) before every timed step; inputs > L2"},
        "gen_latency_s_per_clip": gen_s,
        "e2e": e2e,
        "gpu_launches": launches,
        "clocks": clk,
    }
    if args.impl == "reference":
        out["impl"] = "reference"
        out["gpu_launches"] = None
    if rank == 0:
        print(json.dumps(out))
    barrier()
    if world > 1:
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
