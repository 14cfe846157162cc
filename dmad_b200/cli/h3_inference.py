"""Few-step text-to-audio-video inference with an H3-shaped DMAD student.

Flag-compatible with the reference's ``inference.py`` (inference.py:50-98): --steps, --video-shift,
--audio-shift, --euler, --height/--width/--num-frames, --low-vram [auto|8|12|16|24], --weights-in-ram,
--weights-int8, --lora, --lora-alpha, --seed, --prompt/--prompt-file, --output-dir.

Without real checkpoints (``--model-dir`` absent or ``--random-init``), the network is randomly
initialised with the H3-shaped configuration (``--config 33b`` or ``tiny``) and prompts are replaced by
N(0,1) embeddings of ``--text-tokens`` rows; latents are written instead of decoded video when no VAE
is available.  With ``--model-dir``, ``transformer/config.json`` sets the network's shape and its
``*.safetensors`` shards (this package's parameter names) are loaded into it.  Per-stage peak GPU
memory is logged as the reference does.
"""
from __future__ import annotations

import argparse
import json
import os
import time

import torch

from ..inference.h3 import (H3Geometry, build_packed_sequence, build_row_timesteps, latent_shape_of, rollout,
                            sigma_grid)
from ..inference.text_encoder import read_prompts
from ..models.h3 import H3Config, H3Model


def parse_args(argv=None):
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--model-dir", default=None)
    p.add_argument("--random-init", action="store_true")
    p.add_argument("--config", default="33b", choices=["33b", "tiny"])
    p.add_argument("--lora", default=None)
    p.add_argument("--lora-alpha", type=float, default=None)
    p.add_argument("--prompt", action="append", default=[])
    p.add_argument("--prompt-file", default=None)
    p.add_argument("--text-tokens", type=int, default=256)
    p.add_argument("--output-dir", required=True)
    p.add_argument("--seed", type=int, default=42)
    p.add_argument("--steps", type=int, default=4)
    p.add_argument("--video-shift", type=float, default=12.0)
    p.add_argument("--audio-shift", type=float, default=2.0)
    p.add_argument("--euler", action="store_true")
    p.add_argument("--height", type=int, default=768)
    p.add_argument("--width", type=int, default=1344)
    p.add_argument("--num-frames", type=int, default=124)
    p.add_argument("--low-vram", nargs="?", const="auto", choices=["auto", "8", "12", "16", "24"], default=None)
    p.add_argument("--weights-in-ram", action="store_true",
                   help="with --low-vram: pinned host copies of the streamed weights instead of reading the "
                        "memory-mapped shards on every pass")
    p.add_argument("--weights-int8", action="store_true", help="with --low-vram: int8 per-row streamed weights")
    p.add_argument("--weights-cache", default=None,
                   help="directory of the int8 copy streamed from disk (default ~/.cache/dmad_b200/<id>/int8)")
    p.add_argument("--chunk-rows", type=int, default=None,
                   help="row-chunked blocks: at most this many rows of every intermediate except k / v")
    p.add_argument("--offload", action="store_true", help="same as --low-vram auto")
    # the H3 video / audio VAEs are Diffusers modules that this package does not rebuild; latents are
    # written instead of decoded video, and these two flags only keep reference command lines parsing
    p.add_argument("--vae-offload", action="store_true", help="no effect (the H3 VAEs are external)")
    p.add_argument("--vae-dtype", default="bf16", choices=["bf16", "fp32"], help="no effect (the H3 VAEs are external)")
    p.add_argument("--cp", action="store_true", help="context parallel over all ranks (launch with torchrun): "
                   "every rank holds a slice of the packed sequence")
    p.add_argument("--cp-impl", default="fused", choices=["fused", "nccl", "hybrid"],
                   help="hybrid: Ulysses inside groups of --ulysses-size ranks, ring attention across them "
                        "(for head counts the CP size does not divide)")
    p.add_argument("--ulysses-size", type=int, default=None)
    return p.parse_args(argv)


def main(argv=None):
    args = parse_args(argv)
    prompts = list(args.prompt) + (read_prompts(args.prompt_file) if args.prompt_file else [])
    if not prompts:
        prompts = ["synthetic prompt"]
    os.makedirs(args.output_dir, exist_ok=True)
    if args.offload and not args.low_vram:
        args.low_vram = "auto"
    if args.low_vram:  # GPU size preset -> rows per chunk (every preset gives the same samples up to rounding)
        if args.low_vram == "auto":
            total = torch.cuda.mem_get_info()[1] / 2**30 if torch.cuda.is_available() else 24
            args.low_vram = "8" if total < 11 else "12" if total < 15 else "16" if total < 22 else "24"
        if args.chunk_rows is None:
            args.chunk_rows = {"8": 8192, "12": 8192, "16": 16384, "24": 16384}[args.low_vram]
    cp = None
    if args.cp:
        from ..parallel.cp import make_context_parallel
        from ..parallel.dist import init_distributed
        _, _, device = init_distributed()
        cp = make_context_parallel(impl=args.cp_impl, device=device, ulysses_size=args.ulysses_size)
    else:
        device = torch.device("cuda", torch.cuda.current_device()) if torch.cuda.is_available() else \
            torch.device("cpu")
    rank0 = cp is None or cp.rank == 0
    t0 = time.time()

    def log(msg):
        if rank0:
            print(f"[{time.time() - t0:6.0f}s] {msg}", flush=True)

    def peak(stage):
        if device.type == "cuda":
            log(f"{stage}: peak GPU memory {torch.cuda.max_memory_allocated() / 2**30:.1f} GiB")
            torch.cuda.reset_peak_memory_stats()

    cfg = H3Config() if args.config == "33b" else H3Config(dim=512, num_heads=4, ffn_dim=1024, num_layers=4,
                                                            text_dim=512, time_embed_dim=256)
    tf_dir = None
    if args.model_dir and not args.random_init:
        from ..inference.h3 import config_from_transformer_dir, resolve_transformer_dir
        try:
            tf_dir = resolve_transformer_dir(args.model_dir)
            cfg = config_from_transformer_dir(tf_dir)
        except FileNotFoundError:
            tf_dir = None
    geometry = H3Geometry.from_model_dir(args.model_dir) if (args.model_dir and not args.random_init) else H3Geometry()
    shape = latent_shape_of(args.height, args.width, args.num_frames, geometry)
    vsig, asig = sigma_grid(args.steps, args.video_shift), sigma_grid(args.steps, args.audio_shift)
    g = torch.Generator().manual_seed(args.seed)
    te_dir = os.path.join(args.model_dir, "text_encoder") if args.model_dir else None
    if te_dir and not args.random_init and os.path.isdir(te_dir):
        # the Qwen3-VL conditioner (hidden layer 50, verbatim prompts); freed before the transformer loads
        if args.low_vram:  # decoder layers streamed from the shards, one ahead of compute
            from ..inference.lowmem import LowMemTextEncoder
            enc = LowMemTextEncoder(args.model_dir, device, cache_in_ram=args.weights_in_ram, log=log)
            conds = enc.encode_all(prompts)
            enc.close()
        else:
            from ..inference.text_encoder import Qwen3VLConditioner
            enc = Qwen3VLConditioner.from_pretrained(args.model_dir, device)
            conds = enc.encode_all(prompts)
        del enc
        if device.type == "cuda":
            torch.cuda.empty_cache()
        log(f"encoded {len(conds)} prompt(s)")
    else:
        conds = [{"prompt_embeds": torch.randn(1, args.text_tokens, cfg.text_dim, generator=g).to(torch.bfloat16),
                  "text_token_tags": torch.ones(args.text_tokens, dtype=torch.long)} for _ in prompts]
    layouts = [build_packed_sequence(c["text_token_tags"], shape["latent_frames"], shape["latent_height"],
                                     shape["latent_width"], shape["audio_latents"], geometry.patch_size) for c in conds]
    torch.manual_seed(args.seed)
    source = None
    has_weights = tf_dir is not None and any(tf_dir.glob("*.safetensors"))
    if args.low_vram and has_weights:
        # resident modules loaded now, blocks left on the meta device and streamed from the shards
        from ..inference.lowmem import build_streamed_h3
        model, source = build_streamed_h3(tf_dir, device)
        log(f"resident transformer modules loaded from {tf_dir}; blocks stream from the shards")
    elif device.type == "cuda" and not args.low_vram:
        # build the (33B) model directly on the GPU in bf16: no host copy in fp32
        prev = torch.get_default_dtype()
        torch.set_default_dtype(torch.bfloat16)
        try:
            with torch.device(device):
                model = H3Model(cfg)
        finally:
            torch.set_default_dtype(prev)
    else:
        model = H3Model(cfg).to(torch.bfloat16)
    if has_weights and source is None:
        from ..inference.h3 import load_transformer_weights
        load_transformer_weights(model, tf_dir)
        log(f"transformer weights loaded from {tf_dir}")
    if args.lora:
        from ..lora import attach_lora, lora_rank_alpha, read_lora_file

        pairs, meta = read_lora_file(args.lora)
        rank, alpha = lora_rank_alpha(pairs, meta, args.lora_alpha)
        attach_lora(model, pairs, rank, alpha)
        if source is None:
            model.to(torch.bfloat16)
        log(f"LoRA attached: {len(pairs)} modules, rank {rank}, alpha {alpha:g}")
    model.eval().requires_grad_(False)
    streamed = None
    text_feats = [None] * len(conds)
    tables = None
    if args.low_vram:
        from ..inference.lowmem import LowMemH3, default_cache_dir

        ts = [build_row_timesteps(layouts[0], vsig[s], asig[s])[0] for s in range(args.steps)]
        codec = "int8" if args.weights_int8 else None
        in_ram = args.weights_in_ram or source is None  # a randomly initialised model lives in host memory
        cache_dir = args.weights_cache or (default_cache_dir(tf_dir) if codec and not in_ram else None)
        streamed = LowMemH3(model, device, ts, codec=codec, source=source, cache_in_ram=in_ram, cache_dir=cache_dir,
                            chunk_rows=args.chunk_rows, log=log)
        streamed.precompute_text([c["prompt_embeds"] for c in conds])
        text_feats = [streamed.text_features(c["prompt_embeds"]) for c in conds]
        tables = streamed.tables
        log(f"streaming {streamed.streamer.bytes_per_pass / 2**30:.1f} GiB of weights per model evaluation")
    else:
        model.to(device)
        if cp is not None:
            model.enable_context_parallel(cp)
    outs = []
    for i, (c, lay) in enumerate(zip(conds, layouts)):
        t1 = time.time()
        v, a = rollout(model, c["prompt_embeds"].to(device), lay, shape, geometry, vsig, asig, args.seed, device,
                       renoise=not args.euler, text_features=text_feats[i], adaln_tables_per_step=tables)
        if device.type == "cuda":
            torch.cuda.synchronize()
        log(f"sampled {i + 1}/{len(prompts)} in {time.time() - t1:.1f}s")
        outs.append((v.to(torch.bfloat16), a.to(torch.bfloat16)))
    if streamed is not None:
        streamed.close()
    peak("sampling")
    if rank0:
        for i, ((v, a), prompt) in enumerate(zip(outs, prompts)):
            torch.save({"video_rows": v, "audio_rows": a, "shape": shape},
                       os.path.join(args.output_dir, f"{i:04d}.pt"))
            with open(os.path.join(args.output_dir, f"{i:04d}.txt"), "w", encoding="utf-8") as f:
                f.write(prompt)
        with open(os.path.join(args.output_dir, "settings.json"), "w") as f:
            json.dump({k: v for k, v in vars(args).items() if k != "prompt"}, f, indent=2)
    log("done")
    if cp is not None:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()
    return outs


if __name__ == "__main__":
    main()
