"""Text-to-image evaluation of the SDXL stack: COCO FID, patch FID, CLIP score and LPIPS diversity.

    python -m dmad_b200.tools.coco_eval --images out/ --captions captions.txt --clip-model clip/ \\
        [--ref-stats coco_ref.npz --features inception.pt] [--eval-res 512] [--how-many 10000]

Parity: train/image/main/coco_eval/coco_evaluator.py:36-237 and train/image/main/sdxl/eval_sdxl.py.
* FID: each image is center-cropped on its long edge and resized (``eval_res``, LANCZOS) before the
  feature network; patch FID skips the resize and takes the central 299 x 299 patch of the full image.
  The Frechet distance of the two Gaussian fits is ``samplers.edm.frechet_distance``.  The feature
  network (Inception, or a CLIP image tower) is the caller's ``feature_fn``: no weights ship here.
* CLIP score: mean cosine similarity of image and text embeddings, images center-cropped and resized to
  256 first, captions prefixed with "A photo depicts " (Hessel et al. 2021) and truncated to the text
  tower's length; the CLIP model and processor are Hugging Face ones loaded from local files.
* Diversity: mean pairwise LPIPS of images resized to 512 (``lpips_fn`` is the caller's).
"""
from __future__ import annotations

import argparse
import glob
import os

import numpy as np
import torch
from PIL import Image

from ..samplers.edm import feature_stats, frechet_distance

CLIP_PREFIX = "A photo depicts "


def center_crop_long_edge(img: Image.Image) -> Image.Image:
    s = min(img.size)
    w, h = img.size
    left, top = (w - s) // 2, (h - s) // 2
    return img.crop((left, top, left + s, top + s))


def fid_preprocess(image: np.ndarray, resize: int | None = None, patch: bool = False) -> np.ndarray:
    """uint8 HWC -> uint8 HWC as the FID feature network sees it."""
    img = Image.fromarray(image)
    if patch:
        w, h = img.size
        if min(w, h) < 299:
            raise ValueError("patch FID needs images of at least 299 x 299")
        left, top = (w - 299) // 2, (h - 299) // 2
        img = img.crop((left, top, left + 299, top + 299))
    else:
        img = center_crop_long_edge(img)
        if resize is not None:
            img = img.resize((resize, resize), Image.LANCZOS)
    return np.asarray(img)


def compute_fid(fake_images, feature_fn, ref_stats=None, real_images=None, resize: int | None = None,
                patch: bool = False, batch: int = 64) -> float:
    """FID of uint8 HWC images against reference statistics ``(mu, sigma)`` or against ``real_images``;
    ``feature_fn(uint8 NHWC batch) -> [N, F]`` features."""

    def feats(images):
        out = []
        for s in range(0, len(images), batch):
            chunk = np.stack([fid_preprocess(x, resize, patch) for x in images[s:s + batch]])
            f = feature_fn(chunk)
            out.append(f.detach().cpu().double().numpy() if torch.is_tensor(f) else np.asarray(f, np.float64))
        return np.concatenate(out)

    mu, sig = feature_stats(feats(fake_images))
    if ref_stats is None:
        if real_images is None:
            raise ValueError("need reference statistics or real images")
        ref_stats = feature_stats(feats(real_images))
    return frechet_distance(mu, sig, *ref_stats)


@torch.no_grad()
def clip_score(images, captions, model, processor, how_many: int | None = None, batch: int = 64,
               resize: int = 256, device="cpu") -> float:
    """Mean image-text cosine similarity (Hugging Face ``CLIPModel`` and ``CLIPProcessor``)."""
    n = len(images) if how_many is None else min(how_many, len(images))
    sims = []
    for s in range(0, n, batch):
        ims = [center_crop_long_edge(Image.fromarray(x)).resize((resize, resize), Image.LANCZOS)
               for x in images[s:min(n, s + batch)]]
        txt = [CLIP_PREFIX + c for c in captions[s:min(n, s + batch)]]
        inp = processor(text=txt, images=ims, return_tensors="pt", padding=True, truncation=True)
        inp = {k: v.to(device) for k, v in inp.items()}
        ie = model.get_image_features(pixel_values=inp["pixel_values"])
        te = model.get_text_features(input_ids=inp["input_ids"], attention_mask=inp.get("attention_mask"))
        ie = getattr(ie, "pooler_output", ie)
        te = getattr(te, "pooler_output", te)
        sims.append(torch.nn.functional.cosine_similarity(ie.float(), te.float(), dim=1))
    return float(torch.cat(sims).mean())


@torch.no_grad()
def diversity_score(images, lpips_fn, size: int = 512) -> float:
    """Mean LPIPS over all pairs (images resized to ``size``; ``lpips_fn(a, b)`` on [1, 3, H, W] in [0, 1])."""
    t = [torch.from_numpy(np.asarray(Image.fromarray(x).resize((size, size), Image.LANCZOS))).permute(2, 0, 1)
         .float()[None] / 255.0 for x in images]
    vals = [float(lpips_fn(t[i], t[j])) for i in range(len(t)) for j in range(i + 1, len(t))]
    return float(np.mean(vals)) if vals else 0.0


def load_images(folder: str) -> list[np.ndarray]:
    files = sorted(f for ext in ("png", "jpg", "jpeg") for f in glob.glob(os.path.join(folder, f"*.{ext}")))
    return [np.asarray(Image.open(f).convert("RGB")) for f in files]


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--images", required=True)
    ap.add_argument("--captions", required=True, help="one caption per line, in the images' sorted order")
    ap.add_argument("--clip-model", default=None, help="local Hugging Face CLIP model directory")
    ap.add_argument("--ref-stats", default=None, help="npz with mu / sigma of the reference features")
    ap.add_argument("--features", default=None, help="TorchScript feature network (uint8 NHWC -> [N, F])")
    ap.add_argument("--eval-res", type=int, default=512)
    ap.add_argument("--how-many", type=int, default=None)
    a = ap.parse_args(argv)
    images = load_images(a.images)
    captions = [line.strip() for line in open(a.captions, encoding="utf-8") if line.strip()][:len(images)]
    dev = "cuda" if torch.cuda.is_available() else "cpu"
    res = {}
    if a.ref_stats and a.features:
        ref = np.load(a.ref_stats)
        net = torch.jit.load(a.features, map_location=dev).eval()
        fn = lambda x: net(torch.from_numpy(x).to(dev))  # noqa: E731
        res["fid"] = compute_fid(images, fn, (ref["mu"], ref["sigma"]), resize=a.eval_res)
        res["patch_fid"] = compute_fid(images, fn, (ref["mu_patch"], ref["sigma_patch"]), patch=True) \
            if "mu_patch" in ref else None
    if a.clip_model:
        from transformers import CLIPModel, CLIPProcessor
        model = CLIPModel.from_pretrained(a.clip_model, local_files_only=True).to(dev).eval()
        proc = CLIPProcessor.from_pretrained(a.clip_model, local_files_only=True)
        res["clip_score"] = clip_score(images, captions, model, proc, a.how_many, device=dev)
    print(res)
    return res


if __name__ == "__main__":
    main()
