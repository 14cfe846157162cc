"""Wan text-to-video sampling (4-step distilled students or multi-step teachers), VBench layout.

    torchrun --nproc-per-node 8 -m dmad_b200.cli.wan_sample --distilled --dit_path student.pth \\
        --prompt_json prompts.json --num_samples 5 --output_dir out/

Parity: train/wan/evaluation/vbench_text2video/sample_videos.py:154-666 (``sample_bidirectional``
:213-255, flags :390-425) and the DMAD sample script (train/wan/experiments/dmad/sample.sh).
Prompts are partitioned over data-parallel ranks (``rank // cp`` with ``--cp_size``).  Distilled
sampling runs on the RF grid ``[sigma_max/(sigma_max+1), mid_t..., 0]`` with the re-noise rule
``x = (1 - t') (x - t v) + t' eps`` (fresh seeded noise per step); ``--ode`` uses the Euler rule
``x = x - (t - t') v`` instead; teachers use the shifted grid of ``--num_steps`` with classifier-free
guidance.  Each sample is decoded by the VAE (when ``--vae_path`` is given, or ``--random_vae``)
and written as mp4 (ffmpeg) or ``.npz``, else the latents are saved; ``eval_info.json`` maps
every prompt to its files.
"""
from __future__ import annotations

import argparse
import json
import os

import torch

RES = {"480p": {"16:9": (480, 832), "9:16": (832, 480), "1:1": (624, 624)},
       "720p": {"16:9": (720, 1280), "9:16": (1280, 720), "1:1": (960, 960)}}
_NEG = ("Bright tones, overexposed, static, blurred details, subtitles, style, works, paintings, images, static, "
        "overall gray, worst quality, low quality, JPEG compression residue, ugly, incomplete, extra fingers")


def parse(argv=None):
    p = argparse.ArgumentParser(description="Wan text-to-video sampling")
    p.add_argument("--distilled", action="store_true")
    p.add_argument("--ode", action="store_true", help="deterministic Euler rule instead of re-noising")
    p.add_argument("--prompt_json", default=None, help='JSON list of strings or {"prompt", "augmented_prompt"}')
    p.add_argument("--prompts", default=None, help="text file, one prompt per line")
    p.add_argument("--no_augmented_prompt", action="store_true")
    p.add_argument("--output_dir", default="samples")
    p.add_argument("--num_samples", type=int, default=1)
    p.add_argument("--model_size", choices=["1.3B", "14B"], default="1.3B")
    p.add_argument("--dit_path", default=None, help="release .pth (net.* keys) or a state dict; random init if absent")
    p.add_argument("--vae_path", default=None)
    p.add_argument("--random_vae", action="store_true", help="decode with a random-init VAE (pipeline tests)")
    p.add_argument("--text_encoder_path", default=None)
    p.add_argument("--tokenizer_path", default=None)
    p.add_argument("--num_frames", type=int, default=81)
    p.add_argument("--resolution", default="480p")
    p.add_argument("--aspect_ratio", default="16:9")
    p.add_argument("--fps", type=int, default=16)
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--num_steps", type=int, default=4)
    p.add_argument("--sigma_max", type=float, default=1600.0)
    p.add_argument("--mid_t", type=float, nargs="*", default=None)
    p.add_argument("--guidance_scale", type=float, default=5.0)
    p.add_argument("--negative_prompt", default=_NEG)
    p.add_argument("--timestep_shift", type=float, default=5.0)
    p.add_argument("--cp_size", type=int, default=1)
    p.add_argument("--tiny", action="store_true", help="tiny random model and shapes (smoke tests)")
    return p.parse_args(argv)


def load_prompts(a) -> list[str]:
    if a.prompt_json:
        items = json.load(open(a.prompt_json))
        out = []
        for it in items:
            if isinstance(it, str):
                out.append(it)
            else:
                out.append(it.get("prompt_en") or it.get("prompt") if a.no_augmented_prompt else
                           it.get("augmented_prompt") or it.get("prompt_en") or it.get("prompt"))
        return out
    if a.prompts:
        return [line.strip() for line in open(a.prompts) if line.strip()]
    raise SystemExit("give --prompt_json or --prompts")


def t_grid(a) -> list[float]:
    """RF times from ~1 to 0 (inclusive)."""
    if a.distilled:
        mid = list(a.mid_t) if a.mid_t else [0.9375, 0.8333, 0.625, 0.5, 0.25][: max(0, a.num_steps - 1)]
        return [a.sigma_max / (a.sigma_max + 1.0)] + mid[: a.num_steps - 1] + [0.0]
    from ..samplers import shifted_sigmas
    return shifted_sigmas(a.num_steps, a.timestep_shift).tolist() + [0.0]


@torch.no_grad()
def sample_bidirectional(net, noise, t_steps, ctx, unctx=None, guidance=1.0, ode=False, generator=None):
    x = noise.double() * t_steps[0]
    B = noise.shape[0]
    dt = next(net.parameters()).dtype
    use_cfg = unctx is not None and guidance > 1.0
    for tc, tn in zip(t_steps[:-1], t_steps[1:]):
        ts = torch.full((B, 1), tc * 1000.0, device=noise.device).to(dt).float()
        v = net(x.to(dt), ts, ctx).double()
        if use_cfg:
            vu = net(x.to(dt), ts, unctx).double()
            v = vu + guidance * (v - vu)
        if ode:
            x = x - (tc - tn) * v
        else:
            eps = torch.randn(noise.shape, device=noise.device, generator=generator, dtype=torch.float32).double()
            x = (1 - tn) * (x - tc * v) + tn * eps
    return x.float()


def main(argv=None):
    a = parse(argv)
    from ..models.umt5 import TextEncoder, UMT5Config
    from ..models.wan import WanConfig, WanModel, wan_config
    from ..models.wan_vae import WanVAE, WanVAEModel
    from ..parallel.dist import get_rank, get_world_size, init_distributed

    rank, world, dev = init_distributed()
    dtype = torch.bfloat16 if dev.type == "cuda" else torch.float32
    if a.tiny:
        ncfg = WanConfig(dim=128, ffn_dim=256, num_heads=1, num_layers=2, text_dim=64, freq_dim=64)
        tcfg = UMT5Config(vocab=1000, dim=64, dim_attn=64, dim_ffn=128, num_heads=4, num_layers=2, text_len=16)
        H, W = 64, 64
    else:
        ncfg = wan_config("wan2.1-1.3b" if a.model_size == "1.3B" else "wan2.1-14b")
        tcfg = UMT5Config()
        H, W = RES[a.resolution][a.aspect_ratio]
    net = WanModel(ncfg)
    if a.dit_path:
        sd = torch.load(a.dit_path, map_location="cpu", weights_only=False)
        sd = {k[4:] if k.startswith("net.") else k: v for k, v in sd.items()}
        net.load_state_dict(sd)
    net = net.to(dev, dtype).eval()
    if a.cp_size > 1:
        from ..parallel.cp import ContextParallel
        from ..train.trainer import make_cp_group
        net.enable_context_parallel(ContextParallel(make_cp_group(a.cp_size), device=dev))
    te_model = None
    if a.text_encoder_path:
        from ..models.umt5 import UMT5Encoder
        te_model = UMT5Encoder(tcfg)
        te_model.load_state_dict(torch.load(a.text_encoder_path, map_location="cpu", weights_only=False))
    text = TextEncoder(tcfg, dev, dtype, a.tokenizer_path, te_model)
    vae = None
    if a.vae_path or a.random_vae:
        vm = WanVAEModel(dim=8, z_dim=16, dim_mult=(1, 2, 2, 2), num_res_blocks=1) if a.tiny else WanVAEModel()
        if a.vae_path:
            vm.load_state_dict(torch.load(a.vae_path, map_location="cpu", weights_only=False))
        vae = WanVAE(dev, dtype, vm)
    prompts = load_prompts(a)
    dp_rank, dp_world = rank // a.cp_size, world // a.cp_size
    jobs = [(i, s) for i in range(len(prompts)) for s in range(a.num_samples)][dp_rank::dp_world]
    os.makedirs(a.output_dir, exist_ok=True)
    lat_shape = (1, 16, WanVAE.latent_frames(a.num_frames), H // 8, W // 8)
    grid = t_grid(a)
    info = []
    unctx = None if a.distilled else text.encode([a.negative_prompt])
    for i, s in jobs:
        g = torch.Generator(device=dev).manual_seed(a.seed + 1000 * i + s)
        noise = torch.randn(lat_shape, device=dev, generator=g)
        ctx = text.encode([prompts[i]])
        lat = sample_bidirectional(net, noise, grid, ctx, unctx, 1.0 if a.distilled else a.guidance_scale,
                                   a.ode, g)
        stem = os.path.join(a.output_dir, f"{i:05d}-{s}")
        if get_rank() % a.cp_size == 0:
            if vae is not None:
                from ..inference.h3 import write_mp4
                import numpy as np
                video = vae.decode(lat)[0]                                   # [3, T, H, W] in [-1, 1]
                frames = ((video.permute(1, 2, 3, 0) + 1) * 127.5).round().clamp(0, 255).byte().cpu().numpy()
                path = write_mp4(frames, np.zeros((2, 1), dtype=np.float32), stem + ".mp4")
            else:
                path = stem + ".latent.pt"
                torch.save(lat.cpu(), path)
            info.append({"prompt_index": i, "sample": s, "prompt": prompts[i], "path": os.path.basename(path)})
    if world > 1:
        import torch.distributed as dist
        allinfo = [None] * world
        dist.all_gather_object(allinfo, info)
        info = [x for part in allinfo for x in part]
    if get_rank() == 0:
        with open(os.path.join(a.output_dir, "eval_info.json"), "w") as f:
            json.dump(sorted(info, key=lambda r: (r["prompt_index"], r["sample"])), f, indent=1)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()
    return info


if __name__ == "__main__":
    main()
