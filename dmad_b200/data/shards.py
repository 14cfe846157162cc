"""Tar-shard latent datasets (the Wan DMAD sample layout) split by data-parallel group.

Parity: train/wan/rcm/datasets/webdataset_dmad.py:1-66 and webdataset.py:7-59.  A shard is a
plain tar file whose members are ``<key>.<field>``: ``latent.pt`` (teacher / student-target
latents), ``embed.pt`` (text embeddings), ``prompt.txt`` and, for DMAD, ``real_latent.pt``.
Shards are split over data-parallel ranks (``rank // cp``: all ranks of a context-parallel group
read the same shards) and over loader workers before the shard shuffle, so one pass reads every
shard exactly once; samples pass through a shuffle buffer and are collated into batches with
``dict_collate`` (tensors stacked, strings listed).  Fields are surfaced under the reference's
batch names: latents, t5_text_embeddings, prompts, real_latents.
"""
from __future__ import annotations

import glob
import io
import os
import random
import tarfile

import torch
from torch.utils.data import IterableDataset, get_worker_info

FIELDS = {"latent.pt": "latents", "embed.pt": "t5_text_embeddings", "prompt.txt": "prompts",
          "real_latent.pt": "real_latents"}


def dict_collate(samples: list[dict]) -> dict:
    out = {}
    for k in samples[0]:
        vals = [s[k] for s in samples]
        out[k] = torch.stack(vals) if torch.is_tensor(vals[0]) else vals
    return out


def write_shard(path: str, samples: list[dict]):
    """Write samples ({"__key__": str, field: tensor | str}) as one tar shard (atomic rename)."""
    tmp = path + ".tmp"
    with tarfile.open(tmp, "w") as tf:
        for s in samples:
            key = s["__key__"]
            for field, v in s.items():
                if field == "__key__":
                    continue
                if torch.is_tensor(v):
                    buf = io.BytesIO()
                    torch.save(v, buf)
                    data = buf.getvalue()
                else:
                    data = str(v).encode()
                ti = tarfile.TarInfo(f"{key}.{field}")
                ti.size = len(data)
                tf.addfile(ti, io.BytesIO(data))
    os.replace(tmp, path)


def _decode(field: str, data: bytes):
    if field.endswith(".pt"):
        return torch.load(io.BytesIO(data), map_location="cpu", weights_only=True)
    if field.endswith(".txt"):
        return data.decode()
    return data


def _samples_of(path: str):
    cur_key, cur = None, {}
    with tarfile.open(path, "r") as tf:
        for m in tf:
            if not m.isfile():
                continue
            key, _, field = m.name.partition(".")
            if key != cur_key:
                if cur:
                    yield cur
                cur_key, cur = key, {"__key__": key}
            cur[field] = _decode(field, tf.extractfile(m).read())
    if cur:
        yield cur


class TarShardDataset(IterableDataset):
    def __init__(self, pattern: str, batch_size: int, rank: int = 0, world: int = 1, cp_size: int = 1,
                 shuffle_buffer: int = 1000, seed: int = 0, epochs: int | None = None, partial: bool = False):
        self.shards = sorted(glob.glob(pattern))
        if not self.shards:
            raise FileNotFoundError(f"No files found with pattern '{pattern}'")
        if world % cp_size:
            raise ValueError(f"world_size {world} not divisible by cp_size {cp_size}")
        self.batch_size, self.partial = batch_size, partial
        self.dp_rank, self.dp_world = rank // cp_size, world // cp_size
        self.shuffle_buffer, self.seed, self.epochs = shuffle_buffer, seed, epochs

    def _my_shards(self, epoch: int):
        shards = self.shards[self.dp_rank::self.dp_world] if self.dp_world > 1 else list(self.shards)
        wi = get_worker_info()
        if wi is not None:
            shards = shards[wi.id::wi.num_workers]
        rng = random.Random(self.seed * 1000003 + epoch * 7919 + self.dp_rank)
        rng.shuffle(shards)
        return shards, rng

    def __iter__(self):
        epoch = 0
        while self.epochs is None or epoch < self.epochs:
            shards, rng = self._my_shards(epoch)
            buf, batch = [], []

            def emit(s):
                batch.append({FIELDS.get(k, k): v for k, v in s.items() if k != "__key__"})

            for path in shards:
                for s in _samples_of(path):
                    if self.shuffle_buffer > 1:
                        buf.append(s)
                        if len(buf) < self.shuffle_buffer:
                            continue
                        s = buf.pop(rng.randrange(len(buf)))
                    emit(s)
                    if len(batch) == self.batch_size:
                        yield dict_collate(batch)
                        batch = []
            rng.shuffle(buf)
            for s in buf:
                emit(s)
                if len(batch) == self.batch_size:
                    yield dict_collate(batch)
                    batch = []
            if batch and self.partial:
                yield dict_collate(batch)
            epoch += 1
