"""COCO-style evaluation helpers (parity: train/image/main/coco_eval/coco_evaluator.py): FID / patch-FID
preprocessing and distance, CLIP score with a tiny random Hugging Face CLIP, LPIPS diversity."""
import numpy as np
import pytest
import torch


def test_fid_preprocess_and_distance():
    from dmad_b200.tools.coco_eval import compute_fid, fid_preprocess

    rng = np.random.default_rng(0)
    img = rng.integers(0, 256, size=(320, 400, 3), dtype=np.uint8)
    assert fid_preprocess(img, resize=64).shape == (64, 64, 3)
    p = fid_preprocess(img, patch=True)
    assert p.shape == (299, 299, 3) and np.array_equal(p, img[10:309, 50:349])
    imgs = [rng.integers(0, 256, size=(64, 80, 3), dtype=np.uint8) for _ in range(40)]
    feat = lambda x: torch.from_numpy(x.reshape(len(x), -1)[:, :8].astype(np.float64))  # noqa: E731
    assert abs(compute_fid(imgs, feat, real_images=imgs, resize=32)) < 1e-6
    shifted = [np.clip(x.astype(int) + 40, 0, 255).astype(np.uint8) for x in imgs]
    assert compute_fid(shifted, feat, real_images=imgs, resize=32) > 100


def test_clip_score_matches_manual_cosine():
    transformers = pytest.importorskip("transformers")
    from PIL import Image

    from dmad_b200.tools.coco_eval import CLIP_PREFIX, center_crop_long_edge, clip_score

    cfg = transformers.CLIPConfig(
        text_config=dict(vocab_size=100, hidden_size=32, intermediate_size=64, num_hidden_layers=2,
                         num_attention_heads=2, max_position_embeddings=77),
        vision_config=dict(hidden_size=32, intermediate_size=64, num_hidden_layers=2, num_attention_heads=2,
                           image_size=32, patch_size=8),
        projection_dim=16)
    torch.manual_seed(0)
    model = transformers.CLIPModel(cfg).eval()

    class Proc:  # stands in for CLIPProcessor: characters as token ids, images to [3, 32, 32]
        def __call__(self, text, images, return_tensors, padding, truncation):
            ids = [[1] + [3 + ord(c) % 90 for c in t][:75] + [2] for t in text]
            n = max(len(i) for i in ids)
            ids = torch.tensor([i + [0] * (n - len(i)) for i in ids])
            px = torch.stack([torch.from_numpy(np.asarray(im.resize((32, 32)))).permute(2, 0, 1).float() / 255
                              for im in images])
            return {"input_ids": ids, "attention_mask": (ids > 0).long(), "pixel_values": px}

    rng = np.random.default_rng(1)
    imgs = [rng.integers(0, 256, size=(40, 48, 3), dtype=np.uint8) for _ in range(3)]
    caps = ["a cat", "two dogs", "a red car"]
    s = clip_score(imgs, caps, model, Proc(), batch=2)
    ims = [center_crop_long_edge(Image.fromarray(x)).resize((256, 256), Image.LANCZOS) for x in imgs]
    inp = Proc()([CLIP_PREFIX + c for c in caps], ims, "pt", True, True)
    with torch.no_grad():
        ie = model.get_image_features(pixel_values=inp["pixel_values"])
        te = model.get_text_features(input_ids=inp["input_ids"], attention_mask=inp["attention_mask"])
    ie, te = getattr(ie, "pooler_output", ie), getattr(te, "pooler_output", te)
    ref = torch.nn.functional.cosine_similarity(ie, te, dim=1).mean()
    assert abs(s - float(ref)) < 1e-5


def test_diversity_score():
    from dmad_b200.tools.coco_eval import diversity_score

    imgs = [np.full((16, 16, 3), v, dtype=np.uint8) for v in (0, 128, 255)]
    d = diversity_score(imgs, lambda a, b: (a - b).abs().mean(), size=8)
    assert abs(d - (128 + 255 + 127) / 3 / 255) < 1e-3
