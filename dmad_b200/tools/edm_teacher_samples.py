"""Teacher samples of the EDM stack (the critic's Q images) written as a row-array LMDB.

    python -m dmad_b200.tools.edm_teacher_samples --out teacher_lmdb --num 1000000 [--steps 256] [--seed 10]
        [--teacher ckpt.pt]   (torchrun: every rank generates its slice, rank 0 writes)

Parity: train/image/main/edm/generate_teacher_samples.py:59-307 -- the stochastic Heun sampler (256 steps,
S_churn 40, S_min 0.05, S_max 50, S_noise 1.003), sample i drawn with seed ``seed + i`` and class label
``i mod label_dim``, images quantised as ``clip(x * 127.5 + 128, 0, 255)`` to uint8 and stored with their
labels as rows ``images_<i>`` / ``labels_<i>`` plus the two shape records.
"""
from __future__ import annotations

import argparse

import numpy as np
import torch

from ..data.lmdb_arrays import open_env, write_rows, write_shapes
from ..samplers.edm import edm_heun_sampler


class _PerSampleNoise:
    """randn_like drawing each batch row from its own seeded generator (seed of the sample)."""

    def __init__(self, seeds, device):
        self.gens = [torch.Generator(device).manual_seed(int(s) % (1 << 32)) for s in seeds]

    def __call__(self, x):
        return torch.stack([torch.randn(x.shape[1:], generator=g, device=x.device, dtype=torch.float32)
                            for g in self.gens]).to(x.dtype)


@torch.no_grad()
def generate(net, indices, seed: int = 10, label_dim: int = 1000, steps: int = 256, batch: int = 64, device="cpu"):
    """(uint8 images [n, 3, R, R], int64 labels [n]) of the given sample indices."""
    R, C = net.img_resolution, net.img_channels
    imgs, labs = [], []
    eye = torch.eye(label_dim, device=device)
    for s in range(0, len(indices), batch):
        idx = list(indices[s:s + batch])
        noise = _PerSampleNoise([seed + i for i in idx], device)
        lat = noise(torch.empty(len(idx), C, R, R, device=device))
        lab = torch.tensor([i % label_dim for i in idx], device=device)
        x = edm_heun_sampler(lambda a, sg, c: net(a, sg.expand(a.shape[0]), c), lat, eye[lab], steps=steps,
                             randn_like=noise)
        imgs.append((x * 127.5 + 128).clip(0, 255).to(torch.uint8).cpu())
        labs.append(lab.cpu())
    return torch.cat(imgs).numpy(), torch.cat(labs).numpy().astype(np.int64)


def write_lmdb(env, images, labels, start: int = 0, total: int | None = None):
    write_rows(env, {"images": images, "labels": labels}, start)
    if total is not None:
        write_shapes(env, {"images": images, "labels": labels}, total)


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--out", required=True)
    ap.add_argument("--num", type=int, default=1000000)
    ap.add_argument("--steps", type=int, default=256)
    ap.add_argument("--seed", type=int, default=10)
    ap.add_argument("--batch", type=int, default=64)
    ap.add_argument("--label-dim", type=int, default=1000)
    ap.add_argument("--teacher", default=None, help="state dict of the EDM ImageNet-64 network (config 1)")
    a = ap.parse_args(argv)
    import torch.distributed as dist

    from ..models.edm import config1_unet
    from ..parallel.dist import get_rank, get_world_size, init_distributed

    _, _, dev = init_distributed()
    net = config1_unet(a.label_dim).to(dev).eval()
    if a.teacher:
        net.load_state_dict(torch.load(a.teacher, map_location="cpu"))
    rank, world = get_rank(), get_world_size()
    mine = list(range(rank, a.num, world))
    imgs, labs = generate(net, mine, a.seed, a.label_dim, a.steps, a.batch, dev)
    if world > 1:
        parts = [None] * world
        dist.all_gather_object(parts, (mine, imgs, labs))
    else:
        parts = [(mine, imgs, labs)]
    if rank == 0:
        env = open_env(a.out, readonly=False, map_size=int(1.5 * a.num * imgs[0].nbytes) + (1 << 30))
        for idx, im, lb in parts:
            with env.begin(write=True) as txn:
                for i, x, y in zip(idx, im, lb):
                    txn.put(f"images_{i}_data".encode(), np.ascontiguousarray(x).tobytes())
                    txn.put(f"labels_{i}_data".encode(), np.asarray(y, dtype=np.int64).tobytes())
        write_shapes(env, {"images": imgs, "labels": labs}, a.num)
        print(f"{a.num} teacher samples -> {a.out}")


if __name__ == "__main__":
    main()
