"""Evaluation helpers: VBench aggregation arithmetic and the AVGen-Bench layout."""
import json
import os


def test_vbench_scores(tmp_path):
    from dmad_b200.tools.eval_layout import vbench_scores

    (tmp_path / "a_eval_results.json").write_text(json.dumps({"subject_consistency": [1.0, []],
                                                              "dynamic_degree": [0.5, []],
                                                              "scene": [0.8222, []]}))
    r = vbench_scores(str(tmp_path))
    assert abs(r["quality"] - (1.0 * 1 + 0.5 * 0.5) / 1.5) < 1e-9
    assert abs(r["semantic"] - 1.0) < 1e-9
    assert abs(r["total"] - (4 * r["quality"] + 1.0) / 5) < 1e-12
    assert "color" in r["missing"]


def test_avgenbench_layout(tmp_path):
    from dmad_b200.tools.eval_layout import avgenbench_layout

    rows = [{"category": "music", "content": 'a "cat" / plays', "prompt": "p0"},
            {"category": "speech", "content": "  two   spaces ", "prompt": "p1"}]
    pj = tmp_path / "p.jsonl"
    pj.write_text("\n".join(json.dumps(r) for r in rows))
    out = tmp_path / "out"
    out.mkdir()
    for i in range(2):
        (out / f"{i:04d}.mp4").write_bytes(b"x")
    n = avgenbench_layout(str(pj), str(out), str(tmp_path / "v"), str(tmp_path / "pr"))
    assert n == 2
    assert os.path.exists(tmp_path / "v" / "music" / "a _cat_ _ plays.mp4")
    assert os.path.exists(tmp_path / "v" / "speech" / "two spaces.mp4")
    assert json.load(open(tmp_path / "pr" / "music.json")) == [{"content": rows[0]["content"], "prompt": "p0"}]
