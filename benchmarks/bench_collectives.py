"""Fused compute + collective kernels against their NVLink roofline (2 to 8 GPUs, one process per GPU).

    timeout -k 60 300 python -m torch.distributed.run --nproc-per-node 2 --master-addr 127.0.0.1 \\
        -m benchmarks.bench_collectives --op all

Every figure is timed with CUDA events on the launching stream between barriers and reported as the
maximum over ranks.  Roofline = the bytes that must cross NVLink per GPU and direction divided by
770 GB/s (this pool's measured peer-copy bandwidth per direction).  Compute is far below it for all
three; the AdamW kernel also moves its fp32 shard state through HBM (12 bytes read and written per shard
element), which at 2 GPUs is about two thirds of the NVLink time.

* ``adamw``: ``ShardedAdamW.step`` on N bf16 parameters (one kernel: pull or NVLS ``ld_reduce`` of the
  gradient shard, AdamW on the fp32 shard, push or ``multimem.st`` of the new weights).  Bytes per GPU
  and direction: P2P 2 * 2N (w-1)/w (the shard's gradients in, the new weights out, and the same for
  the peers' reads and writes); NVLS about 2N (reads of this GPU's gradients by the switch, the
  multicast weights coming back).
* ``a2a``: the Ulysses exchange of one Wan-14B CP8 block (q, k, v of 32760 / w tokens, 40 heads of 128:
  ``ContextParallel.seq_to_head``).  Bytes per GPU and direction: 3 * R * D * 2 * (w-1)/w.
* ``ring``: one copy-engine peer copy of a key/value block (2 * R * D bf16).
"""
from __future__ import annotations

import argparse
import json
import os

import torch
import torch.distributed as dist

LINK_GBS = 770.0


def _time(fn, iters, warmup):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    dist.barrier()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(iters):
        fn()
    b.record()
    torch.cuda.synchronize()
    ms = torch.tensor([a.elapsed_time(b) / iters], device="cuda")
    dist.all_reduce(ms, op=dist.ReduceOp.MAX)
    return float(ms)


def bench_adamw(n, iters, warmup, multicast):
    from dmad_b200.parallel.zero import ShardedAdamW

    w = dist.get_world_size()
    p = torch.nn.Parameter(torch.randn(n, device="cuda", dtype=torch.bfloat16) * 0.02)
    opt = ShardedAdamW([p], lr=1e-4, use_multicast=multicast)
    with torch.no_grad():
        p.grad.normal_(0.0, 1e-3)  # the gradient is a view of the optimiser's symmetric flat buffer
    ms = _time(lambda: opt.step(), iters, warmup)
    nv = opt.multicast
    gb = (2 * n if nv else 2 * 2 * n * (w - 1) / w) / 1e9
    roof = gb / LINK_GBS * 1e3
    return {"op": "dp_adamw_fused", "path": "nvls" if nv else "p2p", "params": n, "world": w, "ms": round(ms, 4),
            "nvlink_gb_per_gpu_dir": round(gb, 4), "roofline_ms": round(roof, 4), "frac_of_roofline": round(roof / ms, 3)}


def bench_a2a(tokens, heads, hd, iters, warmup):
    from dmad_b200.parallel.cp import ContextParallel

    w = dist.get_world_size()
    cp = ContextParallel(impl="fused")
    R, D = tokens // w, heads * hd
    rows = torch.randn(R, 3 * D, device="cuda", dtype=torch.bfloat16)
    ms = _time(lambda: cp.seq_to_head(rows, 1, 3, heads, hd), iters, warmup)
    gb = 3 * R * D * 2 * (w - 1) / w / 1e9
    roof = gb / LINK_GBS * 1e3
    return {"op": "cp_seq_to_head_fused", "tokens": tokens, "heads": heads, "world": w, "ms": round(ms, 4),
            "nvlink_gb_per_gpu_dir": round(gb, 4), "roofline_ms": round(roof, 4), "frac_of_roofline": round(roof / ms, 3)}


def bench_ring(tokens, heads, hd, iters, warmup):
    from dmad_b200 import ops
    from dmad_b200.parallel.cp import ContextParallel

    w = dist.get_world_size()
    cp = ContextParallel(impl="ring")
    R, D = tokens // w, heads * hd
    slot, ptrs = cp.slot(2 * R * D)
    slot.normal_()
    cp.sync()
    buf = torch.empty(2 * R * D, device="cuda", dtype=torch.bfloat16)
    src = ptrs[(cp.rank + 1) % w]
    ms = _time(lambda: ops.ext().peer_copy(buf, src, 2 * R * D * 2), iters, warmup)
    cp.sync()
    gb = 2 * R * D * 2 / 1e9
    roof = gb / LINK_GBS * 1e3
    return {"op": "ring_kv_peer_copy", "tokens": tokens, "heads": heads, "world": w, "ms": round(ms, 4),
            "nvlink_gb_per_gpu_dir": round(gb, 4), "roofline_ms": round(roof, 4), "frac_of_roofline": round(roof / ms, 3)}


def bench_nccl_baselines(n, tokens, heads, hd, iters, warmup):
    """The NCCL-only paths the fused kernels replace, on the same bytes: reduce-scatter + all-gather of the
    bf16 gradients / weights (then AdamW would run between them), and the Ulysses all-to-all."""
    w = dist.get_world_size()
    g = torch.randn(n, device="cuda", dtype=torch.bfloat16)
    shard = torch.empty(n // w, device="cuda", dtype=torch.bfloat16)
    full = torch.empty(n, device="cuda", dtype=torch.bfloat16)

    def rs_ag():
        dist.reduce_scatter_tensor(shard, g)
        dist.all_gather_into_tensor(full, shard)

    ms = _time(rs_ag, iters, warmup)
    gb = 2 * 2 * n * (w - 1) / w / 1e9
    out = [{"op": "nccl_reduce_scatter+all_gather", "params": n, "world": w, "ms": round(ms, 4),
            "nvlink_gb_per_gpu_dir": round(gb, 4), "roofline_ms": round(gb / LINK_GBS * 1e3, 4),
            "frac_of_roofline": round(gb / LINK_GBS * 1e3 / ms, 3)}]
    R, D = tokens // w, heads * hd
    src = torch.randn(3 * R * D, device="cuda", dtype=torch.bfloat16)
    dst = torch.empty_like(src)
    ms = _time(lambda: dist.all_to_all_single(dst, src), iters, warmup)
    gb = 3 * R * D * 2 * (w - 1) / w / 1e9
    out.append({"op": "nccl_all_to_all (Ulysses q/k/v bytes)", "tokens": tokens, "heads": heads, "world": w,
                "ms": round(ms, 4), "nvlink_gb_per_gpu_dir": round(gb, 4), "roofline_ms": round(gb / LINK_GBS * 1e3, 4),
                "frac_of_roofline": round(gb / LINK_GBS * 1e3 / ms, 3)})
    return out


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--op", default="all", choices=["all", "adamw", "a2a", "ring", "nccl"])
    ap.add_argument("--params", type=int, default=1 << 28)
    ap.add_argument("--tokens", type=int, default=32760)
    ap.add_argument("--heads", type=int, default=40)
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    a = ap.parse_args(argv)
    from datetime import timedelta
    local = int(os.environ.get("LOCAL_RANK", 0))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))
    res = []
    try:
        if a.op in ("all", "adamw"):
            res.append(bench_adamw(a.params, a.iters, a.warmup, multicast=False))
            res.append(bench_adamw(a.params, a.iters, a.warmup, multicast=True))
        tok = a.tokens // dist.get_world_size() * dist.get_world_size()
        if a.op in ("all", "a2a"):
            res.append(bench_a2a(tok, a.heads, 128, a.iters, a.warmup))
        if a.op in ("all", "ring"):
            res.append(bench_ring(tok, a.heads, 128, a.iters, a.warmup))
        if a.op in ("all", "nccl"):
            res += bench_nccl_baselines(a.params, tok, a.heads, 128, a.iters, a.warmup)
        from dmad_b200.ops import check_device_status
        torch.cuda.synchronize()
        check_device_status()
    finally:
        dist.barrier()
        if dist.get_rank() == 0:
            for r in res:
                print(json.dumps(r), flush=True)
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
