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
