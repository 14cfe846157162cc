"""H3 data preparation and the file pool on CPU: prompt list, pool indices, resumable teacher
samples (tiny model), and FileLatentPool draws (with prefix-bucket lookup)."""
import json
import os

import torch


def test_h3_data_pipeline(tmp_path):
    from dmad_b200.data.h3_pool import FileLatentPool
    from dmad_b200.models.h3 import H3Config, H3Model
    from dmad_b200.tools.h3_data import pool_indices, prompt_list, teacher_data

    caps = [{"clip_id": "c0.mp4", "caption": "a man plays a guitar"}, {"clip_id": "c1.mp4", "caption": "a man  plays a guitar"},
            {"clip_id": "c2.mp4", "caption": "rain on a window"}, {"clip_id": "c3.mp4", "caption": "hi"}]
    (tmp_path / "caps.jsonl").write_text("\n".join(json.dumps(c) for c in caps))
    n = prompt_list(str(tmp_path / "caps.jsonl"), str(tmp_path / "prompts.jsonl"))
    rows = [json.loads(x) for x in open(tmp_path / "prompts.jsonl")]
    assert n == 2 and rows[0]["clip_ids"] == ["c0.mp4", "c1.mp4"]
    real = tmp_path / "real"
    (real / "latents").mkdir(parents=True)
    with open(real / "manifest_rank0.jsonl", "w") as f:
        for cid in ("c0", "c2"):
            f.write(json.dumps({"clip_id": cid, "num_frames": 22}) + "\n")
            torch.save({"video_latent": torch.randn(24, 7, 2, 2), "audio_latent": torch.randn(2, 37, 32)},
                       real / "latents" / f"{cid}.pt")
        f.write(json.dumps({"clip_id": "c9", "skip": "decode error"}) + "\n")
    nclips, idx = pool_indices(str(tmp_path / "prompts.jsonl"), str(real), 22, str(tmp_path / "idx.txt"),
                               num_viz_prompts=0)
    assert nclips == 2 and idx == [0, 1]
    cond_dir = tmp_path / "cache" / "conditions"
    for i in idx:
        d = cond_dir / f"{i:08d}"[-2:]   # prefix bucket layout
        d.mkdir(parents=True, exist_ok=True)
        torch.save({"conditioning": {"positive": {"prompt_embeds": torch.randn(1, 6, 16),
                                                  "text_token_tags": torch.ones(6, dtype=torch.long)}}},
                   d / f"condition_{i:08d}.pt")
    torch.manual_seed(0)
    model = H3Model(H3Config(dim=64, num_heads=1, ffn_dim=96, num_layers=2, refiner_layers=1, text_dim=16,
                             time_embed_dim=32))
    out = teacher_data(str(tmp_path / "cache"), idx, str(tmp_path / "teacher"), steps=2, height=64, width=64,
                       num_frames=22, model=model, device="cpu")
    assert len(out) == 2
    assert teacher_data(str(tmp_path / "cache"), idx, str(tmp_path / "teacher"), model=model, device="cpu") == []
    pool = FileLatentPool(str(real), 22, str(tmp_path / "prompts.jsonl"), str(tmp_path / "cache"),
                          str(tmp_path / "teacher"))
    v, a, tv, ta, cond = pool.draw("cpu")
    assert v.shape == (24, 7, 2, 2) and tv.dim() == 3 and cond["prompt_embeds"].shape == (1, 6, 16)
