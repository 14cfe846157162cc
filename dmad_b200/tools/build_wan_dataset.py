"""Build the Wan DMAD training shards: teacher samples (+ optional real latents) per prompt.

    torchrun --nproc-per-node 8 -m dmad_b200.tools.build_wan_dataset --prompts prompts.txt \\
        --teacher teacher.pth --out /data/wan_dmad --samples-per-shard 64

Parity: train/wan/rcm/datasets/build_synthetic_dataset.py:72-300 (teacher latents from a 100-step
flow Euler sampler, CFG 5, shift 3, seed derived from the prompt index, shards of ``latent.pt``,
``embed.pt``, ``prompt.txt``) and build_real_latents.py:33-196 (``real_latent.pt`` paired by caption).
Prompts are partitioned over ranks; every shard is written to a temporary name and renamed.
``--real-latents dir`` pairs ``<index>.pt`` files from that directory as ``real_latent.pt``.
"""
from __future__ import annotations

import argparse
import os

import torch


def parse(argv=None):
    p = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    p.add_argument("--prompts", required=True, help="text file, one prompt per line")
    p.add_argument("--out", required=True)
    p.add_argument("--teacher", default=None, help="teacher state dict (net.* or plain keys); random init if absent")
    p.add_argument("--model-size", choices=["1.3B", "14B"], default="1.3B")
    p.add_argument("--text-encoder", default=None)
    p.add_argument("--tokenizer", default=None)
    p.add_argument("--real-latents", default=None)
    p.add_argument("--num-frames", type=int, default=81)
    p.add_argument("--height", type=int, default=480)
    p.add_argument("--width", type=int, default=832)
    p.add_argument("--steps", type=int, default=100)
    p.add_argument("--shift", type=float, default=3.0)
    p.add_argument("--guidance", type=float, default=5.0)
    p.add_argument("--negative-prompt", default="")
    p.add_argument("--samples-per-shard", type=int, default=64)
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--tiny", action="store_true", help="tiny random models (pipeline tests)")
    return p.parse_args(argv)


@torch.no_grad()
def main(argv=None):
    a = parse(argv)
    from ..data.shards import write_shard
    from ..models.umt5 import TextEncoder, UMT5Config, UMT5Encoder
    from ..models.wan import WanConfig, WanModel, wan_config
    from ..models.wan_vae import WanVAE
    from ..parallel.dist import init_distributed
    from ..samplers import sample_flow

    rank, world, dev = init_distributed()
    dtype = torch.bfloat16 if dev.type == "cuda" else torch.float32
    if a.tiny:
        ncfg = WanConfig(dim=128, ffn_dim=256, num_heads=1, num_layers=2, text_dim=64, freq_dim=64)
        tcfg = UMT5Config(vocab=1000, dim=64, dim_attn=64, dim_ffn=128, num_heads=4, num_layers=2, text_len=16)
    else:
        ncfg = wan_config("wan2.1-1.3b" if a.model_size == "1.3B" else "wan2.1-14b")
        tcfg = UMT5Config()
    net = WanModel(ncfg)
    if a.teacher:
        sd = torch.load(a.teacher, map_location="cpu", weights_only=False)
        net.load_state_dict({k[4:] if k.startswith("net.") else k: v for k, v in sd.items()})
    net = net.to(dev, dtype).eval()
    te = UMT5Encoder(tcfg)
    if a.text_encoder:
        te.load_state_dict(torch.load(a.text_encoder, map_location="cpu", weights_only=False))
    text = TextEncoder(tcfg, dev, dtype, a.tokenizer, te)
    prompts = [ln.strip() for ln in open(a.prompts) if ln.strip()]
    shape = (1, 16, WanVAE.latent_frames(a.num_frames), a.height // 8, a.width // 8)
    uncond = text.encode([a.negative_prompt])
    os.makedirs(a.out, exist_ok=True)
    mine = list(range(rank, len(prompts), world))
    written = []
    for s0 in range(0, len(mine), a.samples_per_shard):
        samples = []
        for i in mine[s0:s0 + a.samples_per_shard]:
            ctx = text.encode([prompts[i]])
            g = torch.Generator(device=dev).manual_seed(a.seed + i)
            noise = torch.randn(shape, device=dev, generator=g)

            def vel(x, t, c=ctx):
                return net(x.to(dtype), t.reshape(1, 1).to(dtype).float(), c).float()

            x0 = sample_flow(vel, noise, a.steps, a.shift, "euler", a.guidance,
                             (lambda x, t: net(x.to(dtype), t.reshape(1, 1).to(dtype).float(), uncond).float())
                             if a.guidance != 1.0 else None)
            rec = {"__key__": f"{i:08d}", "latent.pt": x0[0].to(torch.bfloat16).cpu(),
                   "embed.pt": ctx[0].cpu(), "prompt.txt": prompts[i]}
            if a.real_latents:
                rp = os.path.join(a.real_latents, f"{i}.pt")
                if os.path.exists(rp):
                    rec["real_latent.pt"] = torch.load(rp, map_location="cpu", weights_only=True)
            samples.append(rec)
        path = os.path.join(a.out, f"shard-r{rank:03d}-{s0 // a.samples_per_shard:05d}.tar")
        write_shard(path, samples)
        written.append(path)
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()
    return written


if __name__ == "__main__":
    main()
