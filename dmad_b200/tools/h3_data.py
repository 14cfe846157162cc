"""H3 DMAD data preparation: prompt list, pool indices and teacher samples.

    python -m dmad_b200.tools.h3_data prompt-list captions.jsonl prompts.jsonl [--min-words 3]
    python -m dmad_b200.tools.h3_data pool-indices --caption-map prompts.jsonl --real-latents real/ --out idx.txt
    python -m dmad_b200.tools.h3_data encode-prompts prompts.jsonl --model-dir H3/ --out cache/ [--indices idx.txt]
        [--shard R/W]          (then: python -m dmad_b200.tools.h3_data merge-prompt-shards cache/)
    python -m dmad_b200.tools.h3_data teacher-data --prompt-cache cache/ --indices idx.txt --out teacher/ \\
        [--model-dir ...] [--shard R/W] [--steps 31] [--video-shift 12] [--audio-shift 3]

Parity: train/h3/data_process/build_prompt_list.py:30-59 (deduplicated caption list with the clip ids of
every caption), build_pool_indices.py:29-47 (caption indices of the clips of the training frame tier, plus
the first visualisation prompts), encode_prompts.py:51-144 (the prompt cache: Qwen3-VL layer-50 conditions
``conditions/condition_<index:08d>.pt`` of the selected prompts, sharded by rank, resumable, one metadata
file per shard merged at the end) and gen_teacher_data.py:48-89 (31-step Euler teacher rollouts, shifts
12 / 3, seed = caption index, resumable, written to a temporary name and renamed).  The outputs are the
files ``data.h3_pool.FileLatentPool`` reads.
"""
from __future__ import annotations

import argparse
import json
import os

import torch


def prompt_list(captions_jsonl: str, out: str, min_words: int = 3) -> int:
    """{"clip_id", "caption"} rows -> {"index", "prompt", "clip_ids"} rows, one per distinct caption."""
    order, clips = [], {}
    for line in open(captions_jsonl, encoding="utf-8"):
        if not line.strip():
            continue
        r = json.loads(line)
        cap = " ".join(str(r.get("caption") or r.get("prompt") or "").split())
        if len(cap.split()) < min_words:
            continue
        if cap not in clips:
            clips[cap] = []
            order.append(cap)
        clips[cap].append(r["clip_id"])
    tmp = out + ".tmp"
    with open(tmp, "w", encoding="utf-8") as f:
        for i, cap in enumerate(order):
            f.write(json.dumps({"index": i, "prompt": cap, "clip_ids": clips[cap]}, ensure_ascii=False) + "\n")
    os.replace(tmp, out)
    return len(order)


def pool_indices(caption_map: str, real_latents: str, num_frames: int, out: str, num_viz_prompts: int = 4):
    from ..data.h3_pool import clip_to_caption, pool_clips

    c2i = clip_to_caption(caption_map)
    idx = set(range(num_viz_prompts))
    n = 0
    for r in pool_clips(real_latents, num_frames):
        n += 1
        if r["clip_id"] in c2i:
            idx.add(c2i[r["clip_id"]])
    with open(out, "w") as f:
        f.write("".join(f"{i}\n" for i in sorted(idx)))
    return n, sorted(idx)


def _write_jsonl(path, rows):
    tmp = f"{path}.tmp{os.getpid()}"
    with open(tmp, "w", encoding="utf-8") as f:
        for r in rows:
            f.write(json.dumps(r, ensure_ascii=False) + "\n")
    os.replace(tmp, path)


def encode_prompts(prompts_path: str, out_dir: str, encoder, indices: list[int] | None = None, shard: str = "",
                   overwrite: bool = False) -> list[dict]:
    """Conditions of the prompts (all, or the caption ``indices``) with ``encoder.encode(prompt)``; files
    that exist are kept unless ``overwrite``.  Returns the metadata rows of this shard."""
    from ..inference.text_encoder import read_prompts

    indexed = list(enumerate(read_prompts(prompts_path)))
    if indices is not None:
        by_idx = dict(indexed)
        indexed = [(i, by_idx[i]) for i in sorted(set(indices))]
    if shard:
        r, w = (int(x) for x in shard.split("/"))
        indexed = indexed[r::w]
    os.makedirs(os.path.join(out_dir, "conditions"), exist_ok=True)
    rows = []
    for index, prompt in indexed:
        rel = os.path.join("conditions", f"condition_{index:08d}.pt")
        path = os.path.join(out_dir, rel)
        if overwrite or not os.path.isfile(path):
            cond = encoder.encode(prompt)
            tmp = f"{path}.tmp{os.getpid()}"
            torch.save({"conditioning": {"positive": cond}, "prompt": prompt, "source_index": index}, tmp)
            os.replace(tmp, path)
        rows.append({"id": index, "caption": prompt, "condition_path": rel})
    name = "metadata.jsonl" if not shard else f"metadata_shard{shard.replace('/', 'of')}.jsonl"
    _write_jsonl(os.path.join(out_dir, name), rows)
    return rows


def merge_prompt_shards(out_dir: str) -> int:
    import glob as _glob

    rows = [json.loads(line) for f in sorted(_glob.glob(os.path.join(out_dir, "metadata_shard*.jsonl")))
            for line in open(f, encoding="utf-8") if line.strip()]
    rows.sort(key=lambda r: r["id"])
    if len({r["id"] for r in rows}) != len(rows):
        raise RuntimeError("duplicate ids across shards")
    _write_jsonl(os.path.join(out_dir, "metadata.jsonl"), rows)
    return len(rows)


@torch.no_grad()
def teacher_data(prompt_cache: str, indices: list[int], out_dir: str, shard: str = "0/1", steps: int = 31,
                 video_shift: float = 12.0, audio_shift: float = 3.0, height: int = 768, width: int = 1344,
                 num_frames: int = 124, model=None, device=None) -> list[str]:
    from ..data.h3_pool import data_file
    from ..inference.h3 import H3Geometry, build_packed_sequence, latent_shape_of, rollout, sigma_grid
    from ..models.h3 import H3Config, H3Model

    r, w = (int(x) for x in shard.split("/"))
    device = torch.device(device) if device is not None else (
        torch.device("cuda", torch.cuda.current_device()) if torch.cuda.is_available() else torch.device("cpu"))
    todo = [i for i in indices[r::w] if not os.path.exists(os.path.join(out_dir, f"{i:08d}.pt"))]
    if not todo:
        return []
    os.makedirs(out_dir, exist_ok=True)
    if model is None:
        model = H3Model(H3Config()).to(device, torch.bfloat16)
    model.eval().requires_grad_(False)
    geo = H3Geometry()
    shape = latent_shape_of(height, width, num_frames, geo)
    vs, as_ = sigma_grid(steps, video_shift), sigma_grid(steps, audio_shift)
    written = []
    for i in todo:
        cond = torch.load(data_file(os.path.join(prompt_cache, "conditions"), f"condition_{i:08d}.pt"),
                          map_location="cpu", weights_only=False)["conditioning"]["positive"]
        lay = build_packed_sequence(cond["text_token_tags"], shape["latent_frames"], shape["latent_height"],
                                    shape["latent_width"], shape["audio_latents"], geo.patch_size)
        v, a = rollout(model, cond["prompt_embeds"].to(device, torch.bfloat16), lay, shape, geo, vs, as_, i, device,
                       renoise=False)
        meta = {"index": i, "seed": i, "steps": steps, "video_shift": video_shift, "audio_shift": audio_shift,
                "num_frames": num_frames}
        out = os.path.join(out_dir, f"{i:08d}.pt")
        tmp = f"{out}.tmp{os.getpid()}"
        torch.save({"video_rows": v.to(torch.bfloat16), "audio_rows": a.to(torch.bfloat16), "meta": meta}, tmp)
        os.replace(tmp, out)
        written.append(out)
    return written


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    sub = ap.add_subparsers(dest="cmd", required=True)
    a = sub.add_parser("prompt-list")
    a.add_argument("captions")
    a.add_argument("out")
    a.add_argument("--min-words", type=int, default=3)
    b = sub.add_parser("pool-indices")
    b.add_argument("--caption-map", required=True)
    b.add_argument("--real-latents", required=True)
    b.add_argument("--num-frames", type=int, default=124)
    b.add_argument("--out", required=True)
    b.add_argument("--num-viz-prompts", type=int, default=4)
    e = sub.add_parser("encode-prompts")
    e.add_argument("prompts")
    e.add_argument("--model-dir", required=True)
    e.add_argument("--out", required=True)
    e.add_argument("--indices", default=None)
    e.add_argument("--shard", default="")
    e.add_argument("--overwrite", action="store_true")
    mg = sub.add_parser("merge-prompt-shards")
    mg.add_argument("out")
    c = sub.add_parser("teacher-data")
    c.add_argument("--prompt-cache", required=True)
    c.add_argument("--indices", required=True)
    c.add_argument("--out", required=True)
    c.add_argument("--shard", default="0/1")
    c.add_argument("--steps", type=int, default=31)
    c.add_argument("--video-shift", type=float, default=12.0)
    c.add_argument("--audio-shift", type=float, default=3.0)
    args = ap.parse_args(argv)
    if args.cmd == "prompt-list":
        print(prompt_list(args.captions, args.out, args.min_words), "captions")
    elif args.cmd == "pool-indices":
        n, idx = pool_indices(args.caption_map, args.real_latents, args.num_frames, args.out, args.num_viz_prompts)
        print(f"{n} clips -> {len(idx)} caption indices -> {args.out}")
    elif args.cmd == "encode-prompts":
        from ..inference.text_encoder import Qwen3VLConditioner
        dev = torch.device("cuda", torch.cuda.current_device()) if torch.cuda.is_available() else torch.device("cpu")
        idx = [int(x) for x in open(args.indices) if x.strip()] if args.indices else None
        rows = encode_prompts(args.prompts, args.out, Qwen3VLConditioner.from_pretrained(args.model_dir, dev), idx,
                              args.shard, args.overwrite)
        print(f"{len(rows)} conditions under {args.out}")
    elif args.cmd == "merge-prompt-shards":
        print(merge_prompt_shards(args.out), "rows merged")
    else:
        idx = [int(x) for x in open(args.indices) if x.strip()]
        out = teacher_data(args.prompt_cache, idx, args.out, args.shard, args.steps, args.video_shift,
                           args.audio_shift)
        print(f"{len(out)} teacher samples written")


if __name__ == "__main__":
    main()
