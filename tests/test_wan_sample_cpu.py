"""The Wan sampling CLI end to end on CPU with a tiny random model: prompt partition, distilled
grid, VAE decode to a file, eval_info.json."""
import json
import os


def test_wan_sample_cli_tiny(tmp_path):
    from dmad_b200.cli.wan_sample import main, t_grid, parse

    pj = tmp_path / "p.json"
    pj.write_text(json.dumps([{"prompt": "a cat", "augmented_prompt": "a fluffy cat"}, "a dog"]))
    info = main(["--tiny", "--distilled", "--prompt_json", str(pj), "--num_samples", "2", "--num_frames", "5",
                 "--output_dir", str(tmp_path / "out"), "--random_vae"])
    assert len(info) == 4
    rec = json.load(open(tmp_path / "out" / "eval_info.json"))
    assert [r["prompt"] for r in rec] == ["a fluffy cat", "a fluffy cat", "a dog", "a dog"]
    for r in rec:
        assert os.path.exists(tmp_path / "out" / r["path"])
    g = t_grid(parse(["--distilled", "--num_steps", "4"]))
    assert len(g) == 5 and g[-1] == 0.0 and abs(g[0] - 1600 / 1601) < 1e-9


def test_build_wan_dataset_tiny(tmp_path):
    """Teacher shards from the dataset builder load through the tar-shard dataset."""
    import torch
    from dmad_b200.data import TarShardDataset
    from dmad_b200.tools.build_wan_dataset import main

    (tmp_path / "p.txt").write_text("a cat\na dog\na bird\n")
    paths = main(["--tiny", "--prompts", str(tmp_path / "p.txt"), "--out", str(tmp_path / "shards"),
                  "--num-frames", "5", "--height", "32", "--width", "32", "--steps", "3",
                  "--samples-per-shard", "2"])
    assert len(paths) == 2
    batches = list(TarShardDataset(str(tmp_path / "shards" / "*.tar"), batch_size=1, shuffle_buffer=1, epochs=1))
    assert len(batches) == 3
    assert batches[0]["latents"].shape == (1, 16, 2, 4, 4) and batches[0]["t5_text_embeddings"].shape == (1, 16, 64)
    assert torch.isfinite(batches[0]["latents"].float()).all()
