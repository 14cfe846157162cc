"""SDXL teacher-sample latents (the critic's Q class) for the captions of a real-latents LMDB.

    python -m dmad_b200.tools.sdxl_teacher_latents generate --real-lmdb real/ --out chunks/ --model-dir sdxl/ \\
        [--shard 0 --num-shards 8] [--batch 16] [--chunk 512] [--steps 50] [--guidance 8] [--seed 20260713]
    python -m dmad_b200.tools.sdxl_teacher_latents merge --out chunks/ --lmdb teacher_lmdb/

Parity: train/image/main/sdxl/generate_teacher_latents.py:1-151 -- for caption i of the real-latents
LMDB (so real and teacher rows share captions), an Euler sampler on the "trailing" timestep spacing of
SDXL's scaled-linear DDPM schedule (50 steps), classifier-free guidance 8 against zero negative
embeddings, noise seeded by the global index of the batch's first sample, latents kept in the scaled VAE
space and stored as fp16; one process per shard writes resumable chunk files that a merge step packs
into an LMDB at the captions' global indices.  The sampler is written here from the Euler method on the
sigma = sqrt((1 - a) / a) parameterisation: the model sees x / sqrt(sigma^2 + 1), the epsilon prediction
is the derivative, and the first latent is drawn at the largest sigma.

The network is this package's ``SDXLUNet``; prompts are encoded by a caller-supplied
``encode(prompts) -> (context [B, 77, 2048], pooled [B, 1280])`` (SDXL's two CLIP text towers, loaded
with transformers from local files by ``clip_text_encoder``).
"""
from __future__ import annotations

import argparse
import glob
import os

import numpy as np
import torch

from ..data.lmdb_arrays import array_shape, open_env, read_string, write_shapes
from ..models.sdxl import ddpm_alphas_cumprod


def euler_trailing_schedule(steps: int, n_train: int = 1000, device="cpu"):
    """(timesteps [steps], sigmas [steps + 1]) of the trailing spacing: t_i = round(T - i T / steps) - 1."""
    t = np.round(np.arange(n_train, 0, -n_train / steps)).astype(np.int64) - 1
    ac = ddpm_alphas_cumprod(n_train).numpy()
    all_sig = ((1 - ac) / ac) ** 0.5
    sig = np.interp(t.astype(np.float64), np.arange(n_train), all_sig)
    return (torch.tensor(t, dtype=torch.float32, device=device),
            torch.tensor(np.concatenate([sig, [0.0]]), dtype=torch.float32, device=device))


@torch.no_grad()
def sample_latents(unet, ctx, pooled, steps: int = 50, guidance: float = 8.0, resolution: int = 1024,
                   generator: torch.Generator | None = None, dtype=None):
    """Teacher latents [B, 4, R/8, R/8] for prompt embeddings (CFG against zero embeddings)."""
    dev = ctx.device
    dtype = dtype or next(unet.parameters()).dtype
    B = ctx.shape[0]
    ts, sig = euler_trailing_schedule(steps, device=dev)
    r = resolution // 8
    x = torch.randn((B, 4, r, r), generator=generator, device=generator.device if generator else dev,
                    dtype=torch.float32).to(dev) * sig[0]
    ids = torch.tensor([resolution, resolution, 0, 0, resolution, resolution], device=dev,
                       dtype=torch.float32).expand(B, 6)
    ctx2 = torch.cat([torch.zeros_like(ctx), ctx]).to(dtype)
    pooled2 = torch.cat([torch.zeros_like(pooled), pooled]).to(dtype)
    ids2 = torch.cat([ids, ids])
    for i in range(steps):
        xin = (x / (sig[i] ** 2 + 1) ** 0.5).to(dtype)
        eps = unet(torch.cat([xin, xin]), ts[i].expand(2 * B), ctx2, ids2, pooled2).float()
        eu, ec = eps.chunk(2)
        eps = eu + guidance * (ec - eu)
        x = x + eps * (sig[i + 1] - sig[i])
    return x


def load_prompts(real_lmdb, num_samples: int | None = None) -> list[str]:
    env = open_env(real_lmdb) if isinstance(real_lmdb, str) else real_lmdb
    n = array_shape(env, "latents")[0]
    n = n if num_samples is None else min(n, num_samples)
    return [read_string(env, "prompts", i) for i in range(n)]


def chunk_path(out_dir: str, shard: int, idx: int) -> str:
    return os.path.join(out_dir, f"shard{shard:02d}_chunk{idx:05d}.npz")


def _complete(path: str, n: int) -> bool:
    try:
        with np.load(path, allow_pickle=True) as z:
            return z["latents"].shape[0] == n
    except Exception:  # noqa: BLE001 - missing or partial file
        return False


def generate(unet, encode, prompts: list[str], out_dir: str, shard: int = 0, num_shards: int = 1, batch: int = 16,
             chunk: int = 512, steps: int = 50, guidance: float = 8.0, resolution: int = 1024,
             seed: int = 20260713, device="cpu") -> list[str]:
    """Writes this shard's chunk files (skipping complete ones); returns the paths written."""
    os.makedirs(out_dir, exist_ok=True)
    mine = list(range(shard, len(prompts), num_shards))
    written = []
    for ci in range(0, -(-len(mine) // chunk)):
        path = chunk_path(out_dir, shard, ci)
        idxs = mine[ci * chunk:(ci + 1) * chunk]
        if _complete(path, len(idxs)):
            continue
        lats = []
        for b0 in range(0, len(idxs), batch):
            bidx = idxs[b0:b0 + batch]
            ctx, pooled = encode([prompts[i] for i in bidx])
            g = torch.Generator(device="cpu").manual_seed(seed + bidx[0])
            lats.append(sample_latents(unet, ctx.to(device), pooled.to(device), steps, guidance, resolution, g)
                        .to(torch.float16).cpu().numpy())
        tmp = path + ".tmp.npz"
        np.savez(tmp, latents=np.concatenate(lats), prompt_idx=np.array(idxs, dtype=np.int64),
                 prompts=np.array([prompts[i] for i in idxs], dtype=object))
        os.replace(tmp, path)
        written.append(path)
    return written


def merge(out_dir: str, env) -> int:
    """Packs every chunk into the LMDB environment at the captions' global indices."""
    chunks = sorted(glob.glob(os.path.join(out_dir, "shard*_chunk*.npz")))
    if not chunks:
        raise FileNotFoundError(f"no chunks in {out_dir}")
    total, shape = 0, None
    for c in chunks:
        with np.load(c, allow_pickle=True) as z:
            total += z["latents"].shape[0]
            shape = z["latents"].shape[1:]
    seen = np.zeros(total, dtype=bool)
    with env.begin(write=True) as txn:
        for c in chunks:
            with np.load(c, allow_pickle=True) as z:
                for lat, text, gi in zip(z["latents"], z["prompts"], z["prompt_idx"]):
                    gi = int(gi)
                    if seen[gi]:
                        raise RuntimeError(f"duplicate index {gi} in {c}")
                    seen[gi] = True
                    txn.put(f"latents_{gi}_data".encode(), np.asarray(lat, np.float16).tobytes())
                    txn.put(f"prompts_{gi}_data".encode(), str(text).encode())
    if not seen.all():
        raise RuntimeError(f"{int((~seen).sum())} indices missing from the chunks")
    write_shapes(env, {"latents": np.empty((total,) + tuple(shape), np.float16)}, total)
    return total


def clip_text_encoder(model_dir: str, device, dtype=torch.float16):
    """SDXL's prompt encoder from a local stable-diffusion-xl-base folder: penultimate hidden states of
    both CLIP text towers concatenated (77 x 2048) and the projected pooled output of the second (1280)."""
    from transformers import CLIPTextModel, CLIPTextModelWithProjection, CLIPTokenizer

    tok1 = CLIPTokenizer.from_pretrained(os.path.join(model_dir, "tokenizer"), local_files_only=True)
    tok2 = CLIPTokenizer.from_pretrained(os.path.join(model_dir, "tokenizer_2"), local_files_only=True)
    te1 = CLIPTextModel.from_pretrained(os.path.join(model_dir, "text_encoder"), torch_dtype=dtype,
                                        local_files_only=True).to(device).eval()
    te2 = CLIPTextModelWithProjection.from_pretrained(os.path.join(model_dir, "text_encoder_2"), torch_dtype=dtype,
                                                      local_files_only=True).to(device).eval()

    @torch.no_grad()
    def encode(prompts):
        outs, pooled = [], None
        for tok, te in ((tok1, te1), (tok2, te2)):
            ids = tok(prompts, padding="max_length", max_length=tok.model_max_length, truncation=True,
                      return_tensors="pt").input_ids.to(device)
            o = te(ids, output_hidden_states=True)
            outs.append(o.hidden_states[-2])
            if te is te2:
                pooled = o.text_embeds
        return torch.cat(outs, dim=-1), pooled

    return encode


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    sub = ap.add_subparsers(dest="cmd", required=True)
    g = sub.add_parser("generate")
    g.add_argument("--real-lmdb", required=True)
    g.add_argument("--out", required=True)
    g.add_argument("--model-dir", required=True, help="local stable-diffusion-xl-base-1.0 folder")
    g.add_argument("--unet", default=None, help="state dict of the SDXL U-Net (default: <model-dir>/unet.pt)")
    g.add_argument("--num-samples", type=int, default=500000)
    g.add_argument("--shard", type=int, default=0)
    g.add_argument("--num-shards", type=int, default=8)
    g.add_argument("--batch", type=int, default=16)
    g.add_argument("--chunk", type=int, default=512)
    g.add_argument("--steps", type=int, default=50)
    g.add_argument("--guidance", type=float, default=8.0)
    g.add_argument("--resolution", type=int, default=1024)
    g.add_argument("--seed", type=int, default=20260713)
    m = sub.add_parser("merge")
    m.add_argument("--out", required=True)
    m.add_argument("--lmdb", required=True)
    a = ap.parse_args(argv)
    if a.cmd == "merge":
        env = open_env(a.lmdb, readonly=False)
        print(merge(a.out, env), "teacher latents ->", a.lmdb)
        return
    from ..models.sdxl import SDXLUNet

    dev = torch.device("cuda" if torch.cuda.is_available() else "cpu")
    dtype = torch.float16 if dev.type == "cuda" else torch.float32
    unet = SDXLUNet().to(dev, dtype).eval()
    unet.load_state_dict(torch.load(a.unet or os.path.join(a.model_dir, "unet.pt"), map_location="cpu"))
    prompts = load_prompts(a.real_lmdb, a.num_samples)
    paths = generate(unet, clip_text_encoder(a.model_dir, dev, dtype), prompts, a.out, a.shard, a.num_shards, a.batch,
                     a.chunk, a.steps, a.guidance, a.resolution, a.seed, dev)
    print(f"shard {a.shard}: {len(paths)} chunk(s) written")


if __name__ == "__main__":
    main()
