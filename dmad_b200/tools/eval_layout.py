"""Evaluation helpers: VBench score aggregation and the AVGen-Bench file layout.

* ``vbench_scores(result_dir)`` -- reads VBench's ``*_eval_results.json`` files, min-max normalises
  the 16 dimensions with VBench's published ranges, and combines them into the Quality (7 dims,
  dynamic degree weighted 1/2), Semantic (9 dims) and Total (4:1) scores.  Parity:
  train/wan/evaluation/vbench_text2video/cal_scores.py.
* ``avgenbench_layout(prompts_jsonl, output_dir, videos_dir, prompts_dir)`` -- places the
  ``<i:04d>.mp4`` outputs of the H3 inference CLI where AVGen-Bench looks for them
  (``<videos_dir>/<category>/<file name from the prompt content>.mp4``) and writes its
  per-category prompt lists.  Parity: train/h3/evaluation/avgenbench/layout.py.

    python -m dmad_b200.tools.eval_layout vbench <result_dir>
    python -m dmad_b200.tools.eval_layout avgenbench prompts.jsonl outputs/ videos/ [--prompts-dir d] [--copy]
"""
from __future__ import annotations

import argparse
import json
import os
import re
import shutil

# VBench dimensions, weights and normalisation ranges (the benchmark's published scoring)
QUALITY = {"subject consistency": (0.1462, 1.0, 1.0), "background consistency": (0.2615, 1.0, 1.0),
           "temporal flickering": (0.6293, 1.0, 1.0), "motion smoothness": (0.706, 0.9975, 1.0),
           "aesthetic quality": (0.0, 1.0, 1.0), "imaging quality": (0.0, 1.0, 1.0),
           "dynamic degree": (0.0, 1.0, 0.5)}
SEMANTIC = {"object class": (0.0, 1.0, 1.0), "multiple objects": (0.0, 1.0, 1.0), "human action": (0.0, 1.0, 1.0),
            "color": (0.0, 1.0, 1.0), "spatial relationship": (0.0, 1.0, 1.0), "scene": (0.0, 0.8222, 1.0),
            "appearance style": (0.0009, 0.2855, 1.0), "temporal style": (0.0, 0.364, 1.0),
            "overall consistency": (0.0, 0.364, 1.0)}


def vbench_scores(result_dir: str) -> dict:
    raw = {}
    for name in sorted(os.listdir(result_dir)):
        if name.endswith("_eval_results.json"):
            for k, v in json.load(open(os.path.join(result_dir, name))).items():
                raw[k.replace("_", " ")] = v[0] if isinstance(v, list) and v else v
    out = {"dims": {}}

    def group(table):
        num = den = 0.0
        for d, (lo, hi, w) in table.items():
            if d not in raw or not isinstance(raw[d], (int, float)):
                continue
            n = min(1.0, max(0.0, (raw[d] - lo) / (hi - lo))) if hi > lo else 0.0
            out["dims"][d] = {"raw": raw[d], "norm": n, "weight": w}
            num += n * w
            den += w
        return num / den if den else 0.0

    out["quality"] = group(QUALITY)
    out["semantic"] = group(SEMANTIC)
    out["total"] = (4 * out["quality"] + out["semantic"]) / 5
    out["missing"] = [d for d in list(QUALITY) + list(SEMANTIC) if d not in out["dims"]]
    return out


def _safe_name(text: str, max_len: int = 180) -> str:
    """The file name AVGen-Bench derives from a prompt's content."""
    s = re.sub(r'[/\\:*?"<>|\n\r\t]', "_", str(text).strip())
    s = re.sub(r"\s+", " ", s).strip() or "untitled"
    return s[:max_len].rstrip() if len(s) > max_len else s


def avgenbench_layout(prompts_jsonl: str, output_dir: str, videos_dir: str, prompts_dir: str | None = None,
                      copy: bool = False) -> int:
    rows = [json.loads(ln) for ln in open(prompts_jsonl, encoding="utf-8") if ln.strip()]
    missing = [i for i in range(len(rows)) if not os.path.isfile(os.path.join(output_dir, f"{i:04d}.mp4"))]
    if missing:
        raise FileNotFoundError(f"{len(missing)} of {len(rows)} videos missing in {output_dir}, e.g. {missing[:5]}")
    cats: dict = {}
    for i, r in enumerate(rows):
        src = os.path.abspath(os.path.join(output_dir, f"{i:04d}.mp4"))
        dst = os.path.join(videos_dir, r["category"], _safe_name(r["content"]) + ".mp4")
        os.makedirs(os.path.dirname(dst), exist_ok=True)
        if os.path.lexists(dst):
            os.remove(dst)
        (shutil.copyfile if copy else os.symlink)(src, dst)
        cats.setdefault(r["category"], []).append({"content": r["content"], "prompt": r["prompt"]})
    if prompts_dir:
        os.makedirs(prompts_dir, exist_ok=True)
        for c, items in cats.items():
            with open(os.path.join(prompts_dir, f"{c}.json"), "w", encoding="utf-8") as f:
                json.dump(items, f, ensure_ascii=False, indent=2)
    return len(rows)


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    sub = ap.add_subparsers(dest="cmd", required=True)
    v = sub.add_parser("vbench")
    v.add_argument("result_dir")
    a = sub.add_parser("avgenbench")
    a.add_argument("prompts_jsonl")
    a.add_argument("output_dir")
    a.add_argument("videos_dir")
    a.add_argument("--prompts-dir")
    a.add_argument("--copy", action="store_true")
    args = ap.parse_args(argv)
    if args.cmd == "vbench":
        r = vbench_scores(args.result_dir)
        for d, x in r["dims"].items():
            print(f"{d:<26s} {x['raw']:8.4f} {x['norm']:8.4f} {x['weight']:4.1f}")
        print(f"quality {r['quality']:.4f} semantic {r['semantic']:.4f} total {r['total']:.4f}")
        return r
    n = avgenbench_layout(args.prompts_jsonl, args.output_dir, args.videos_dir, args.prompts_dir, args.copy)
    print(f"{n} videos -> {args.videos_dir}")
    return n


if __name__ == "__main__":
    main()
