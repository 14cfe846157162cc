"""The H3 DMAD data pool on disk: encoded real clips, caption-indexed prompt conditions and teacher samples.

Parity: ``RealLatentPool`` (train/h3/lightx2v_train/trainers/dmd/minimax_h3_dmad_trainer.py:75-132) and
the data layout written by train/h3/data_process/*.py:

    <real>/manifest_rank*.jsonl        {"clip_id", "num_frames"} per encoded clip ("skip" marks failures)
    <real>/latents/<clip_id>.pt         {"video_latent": [24, T', H', W'], "audio_latent": [2, n, 32]}
    <caption_map>                       {"index", "clip_ids": [...]} per caption
    <prompt_cache>/conditions/condition_<index:08d>.pt   {"conditioning": {"positive": {...}}}
    <teacher>/<index:08d>.pt            {"video_rows": [1, Rv, 96], "audio_rows": [1, Ra, 32], "meta"}

A file may also sit in a bucket directory named by the last two characters of its stem (the released
prompt cache is laid out that way).  ``draw`` returns (real video, real audio, teacher video rows,
teacher audio rows, condition) of one random clip with a caption and a teacher sample; the pool
refuses to start when clips lack captions or teacher samples.
"""
from __future__ import annotations

import glob
import json
import os
import random

import torch


def data_file(directory: str, name: str) -> str:
    """``directory/name`` or, when absent, ``directory/<last two chars of stem>/name``."""
    p = os.path.join(directory, name)
    if os.path.isfile(p):
        return p
    return os.path.join(directory, os.path.splitext(name)[0][-2:], name)


def clip_to_caption(caption_map: str) -> dict:
    out = {}
    for line in open(caption_map, encoding="utf-8"):
        if line.strip():
            r = json.loads(line)
            for c in r["clip_ids"]:
                out.setdefault(c.rsplit(".", 1)[0], int(r["index"]))
    return out


def pool_clips(real_dir: str, num_frames: int):
    for mf in sorted(glob.glob(os.path.join(real_dir, "manifest_rank*.jsonl"))):
        for line in open(mf, encoding="utf-8"):
            if line.strip():
                r = json.loads(line)
                if "skip" not in r and r.get("num_frames") == num_frames:
                    yield r


class FileLatentPool:
    def __init__(self, real_dir: str, num_frames: int, caption_map: str, prompt_cache: str, teacher_dir: str,
                 seed: int = 0):
        if not glob.glob(os.path.join(real_dir, "manifest_rank*.jsonl")):
            raise FileNotFoundError(f"no manifest_rank*.jsonl under {real_dir}")
        c2i = clip_to_caption(caption_map)
        self.cond_dir = os.path.join(prompt_cache, "conditions")
        self.teacher_dir = teacher_dir
        self.paths, self.idx = [], []
        unmapped = no_teacher = 0
        for r in pool_clips(real_dir, num_frames):
            i = c2i.get(r["clip_id"])
            if i is None:
                unmapped += 1
                continue
            if not os.path.isfile(data_file(teacher_dir, f"{i:08d}.pt")):
                no_teacher += 1
                continue
            self.idx.append(i)
            self.paths.append(data_file(os.path.join(real_dir, "latents"), f"{r['clip_id']}.pt"))
        if not self.paths:
            raise RuntimeError(f"real pool empty for num_frames={num_frames} under {real_dir}")
        if unmapped:
            raise RuntimeError(f"{unmapped} real clips have no caption in {caption_map}")
        if no_teacher:
            raise RuntimeError(f"{no_teacher} real clips have no teacher sample under {teacher_dir}")
        self.rng = random.Random(seed)

    def __len__(self):
        return len(self.paths)

    def _condition(self, i):
        d = torch.load(data_file(self.cond_dir, f"condition_{self.idx[i]:08d}.pt"), map_location="cpu",
                       weights_only=False)
        return d["conditioning"]["positive"]

    def draw_condition(self):
        return self._condition(self.rng.randrange(len(self.paths)))

    def draw(self, device, dtype=torch.float32):
        i = self.rng.randrange(len(self.paths))
        d = torch.load(self.paths[i], map_location="cpu", weights_only=False)
        t = torch.load(data_file(self.teacher_dir, f"{self.idx[i]:08d}.pt"), map_location="cpu", weights_only=False)
        return (d["video_latent"].to(device, dtype), d["audio_latent"].to(device, dtype),
                t["video_rows"].to(device, dtype), t["audio_rows"].to(device, dtype), self._condition(i))
