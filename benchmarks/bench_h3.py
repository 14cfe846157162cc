"""MiniMax-H3-shaped 33B audio-video DiT sampling (random-init weights), bf16.

    python -m benchmarks.bench_h3 --mode resident --steps 4                     # 1 GPU, weights resident
    torchrun --nproc-per-node 8 -m benchmarks.bench_h3 --mode cp --steps 4      # context parallel over 8 GPUs
    python -m benchmarks.bench_h3 --mode lowvram --budget-gib 16 --steps 4      # 1 GPU, blocks streamed

One video = a 4- (or 8-) step rollout of the student on a 5 s 1344x768 clip (124 frames) plus stereo audio,
packed as the H3 pipeline packs it (text | audio | video rows, ~38k tokens).  Timed with CUDA events after
a warm-up rollout, max over ranks; "s per evaluation" = rollout time / steps.  The reference publishes
9 s per evaluation and 37 s per 4-step video on one H200, and peak memory 5.9 GiB while sampling with
``--low-vram`` (README.md:205, 242-251).

``lowvram`` runs the ``--low-vram 16`` path of the CLI: every block streamed host -> device through the
native engine (pinned RAM copies: the random weights are generated block by block on the GPU and moved
to pinned host memory, no checkpoint is read), adaLN tables and the text refiner precomputed, blocks
row-chunked; it reports the peak device memory of the sampling phase against the budget and the H2D
bytes streamed per evaluation.
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


def _init_weights_(module, std=0.02, gen=None):
    with torch.no_grad():
        for p in module.parameters():
            if p.dim() >= 2:
                p.normal_(0.0, std, generator=gen)
            else:
                p.normal_(0.0, 0.01, generator=gen)


def _case(args, cfg):
    from dmad_b200.inference.h3 import H3Geometry, build_packed_sequence, latent_shape_of, sigma_grid

    geo = H3Geometry()
    shape = latent_shape_of(args.height, args.width, args.num_frames, geo)
    tags = torch.ones(args.text_tokens, dtype=torch.long)
    lay = build_packed_sequence(tags, shape["latent_frames"], shape["latent_height"], shape["latent_width"],
                                shape["audio_latents"], geo.patch_size)
    vs, as_ = sigma_grid(args.steps, 12.0), sigma_grid(args.steps, 2.0)
    pe = torch.randn(1, args.text_tokens, cfg.text_dim, generator=torch.Generator().manual_seed(3)).to(torch.bfloat16)
    return geo, shape, lay, vs, as_, pe


def sigma_grid_n(steps):
    from dmad_b200.inference.h3 import sigma_grid

    return sigma_grid(steps, 12.0), sigma_grid(steps, 2.0)


def main(argv=None):
    ap = argparse.ArgumentParser(description="config-5 H3 33B-shaped sampling")
    ap.add_argument("--mode", default="resident", choices=["resident", "cp", "lowvram"])
    ap.add_argument("--steps", default="4", help="comma-separated step counts, each timed (e.g. 4,8)")
    ap.add_argument("--runs", type=int, default=1)
    ap.add_argument("--layers", type=int, default=None, help="debug only: fewer blocks (invalid for the headline)")
    ap.add_argument("--height", type=int, default=768)
    ap.add_argument("--width", type=int, default=1344)
    ap.add_argument("--num-frames", type=int, default=124)
    ap.add_argument("--text-tokens", type=int, default=256)
    ap.add_argument("--budget-gib", type=float, default=16.0)
    ap.add_argument("--cp-impl", default="fused", choices=["fused", "nccl"])
    a = ap.parse_args(argv)
    from dmad_b200.inference.h3 import build_row_timesteps, rollout
    from dmad_b200.models.h3 import H3Config, H3Model

    step_counts = [int(x) for x in str(a.steps).split(",")]
    a.steps = max(step_counts)
    if a.mode == "lowvram" and len(step_counts) > 1:
        raise SystemExit("lowvram precomputes the adaLN tables of one step count: pass one --steps value")
    cfg = H3Config() if a.layers is None else H3Config(num_layers=a.layers)
    cp = None
    if a.mode == "cp":
        from dmad_b200.parallel.cp import make_context_parallel
        from dmad_b200.parallel.dist import init_distributed
        _, _, device = init_distributed(timeout_s=600)
        cp = make_context_parallel(impl=a.cp_impl, device=device)
    else:
        device = torch.device("cuda", 0)
        torch.cuda.set_device(device)
    rank0 = cp is None or cp.rank == 0
    geo, shape, lay, vs, as_, pe = _case(a, cfg)
    torch.manual_seed(0)
    gen = torch.Generator(device=device).manual_seed(0)
    streamed = None
    text_features = tables = None
    t_build = time.time()
    if a.mode == "lowvram":
        from dmad_b200.inference.lowmem import LowMemH3, _buffers_to, empty_parameters

        with empty_parameters():
            model = H3Model(cfg).to(torch.bfloat16)
        # resident modules on the device; blocks materialised one at a time on the device, then pinned host
        for name, mod in model.named_children():
            if name == "transformer_blocks":
                continue
            mod.to_empty(device=device)
            _init_weights_(mod, gen=gen)
        for b in model.transformer_blocks:
            b.to_empty(device=device)
            _init_weights_(b, gen=gen)
            for m in b.modules():
                for k, p in list(m._parameters.items()):
                    if p is not None:
                        m._parameters[k] = torch.nn.Parameter(p.detach().cpu().pin_memory(), requires_grad=False)
            _buffers_to(b, "cpu")
        torch.cuda.empty_cache()
        model.eval().requires_grad_(False)
        ts = [build_row_timesteps(lay, vs[s], as_[s])[0] for s in range(a.steps)]
        chunk = {8: 8192, 12: 8192, 16: 16384, 24: 16384}.get(int(a.budget_gib), 16384)
        torch.cuda.reset_peak_memory_stats()
        streamed = LowMemH3(model, device, ts, cache_in_ram=True, chunk_rows=chunk)
        streamed.precompute_text([pe])
        text_features = streamed.text_features(pe)
        tables = streamed.tables
    else:
        prev = torch.get_default_dtype()
        torch.set_default_dtype(torch.bfloat16)
        try:
            with torch.device(device):
                model = H3Model(cfg)
        finally:
            torch.set_default_dtype(prev)
        _init_weights_(model, gen=gen)
        if cp is not None:
            from dmad_b200.parallel.dist import broadcast_module
            broadcast_module(model)
            model.enable_context_parallel(cp)
        model.eval().requires_grad_(False)
    build_s = time.time() - t_build

    results = []
    for steps in step_counts:
        vs_n, as_n = sigma_grid_n(steps)
        tab = None if tables is None else tables[:steps]

        def one():
            return rollout(model, pe.to(device), lay, shape, geo, vs_n, as_n, 7, device, text_features=text_features,
                           adaln_tables_per_step=tab)

        with torch.no_grad():
            one()  # warm-up rollout
            torch.cuda.synchronize()
            torch.cuda.reset_peak_memory_stats()
            times = []
            for _ in range(a.runs):
                if cp is not None:
                    torch.distributed.barrier()
                s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                s.record()
                one()
                e.record()
                e.synchronize()
                times.append(s.elapsed_time(e) / 1000.0)
        t = min(times)
        peak = torch.cuda.max_memory_allocated() / 2 ** 30
        if cp is not None:
            v = torch.tensor([t, peak], device=device, dtype=torch.float64)
            torch.distributed.all_reduce(v, op=torch.distributed.ReduceOp.MAX)
            t, peak = float(v[0]), float(v[1])
        results.append({"steps": steps, "s_per_video": t, "s_per_evaluation": t / steps, "peak_sampling_gib": round(peak, 2)})
    out = {"metric": "H3 33B-shaped sampling: s per video and s per model evaluation (device-timed, max over ranks)",
           "mode": a.mode, "results": results, "tokens": int(lay.sequence_length),
           "gpus": cp.world if cp is not None else 1, "build_s": round(build_s, 1),
           "config": {"model": f"H3-shaped DiT, {cfg.num_layers} blocks, hidden {cfg.dim}, ffn {cfg.ffn_dim}",
                      "video": f"{a.num_frames} frames at {a.height}x{a.width}", "text_tokens": a.text_tokens,
                      "dtype": "bf16", "weights": "random init"},
           "reference_published": {"s_per_evaluation_h200": 9.0, "s_per_video_4step_h200": 37.0,
                                   "lowvram_peak_sampling_gib": 5.9}}
    if streamed is not None:
        st = streamed.streamer.stats()
        out["budget_gib"] = a.budget_gib
        out["h2d_gb_per_evaluation"] = round(streamed.streamer.bytes_per_pass / 1e9, 2)
        out["engine_host_wait_s"] = round(st["host_wait_s"], 3)
        streamed.close()
    if rank0:
        print(json.dumps(out), flush=True)
    if cp is not None:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
