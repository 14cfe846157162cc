"""H3 transformer folder loading: config.json -> H3Config, safetensors shards (with an index) -> weights."""
import json

import pytest
import torch

from dmad_b200.inference.h3 import (config_from_transformer_dir, load_transformer, load_transformer_weights,
                                    resolve_transformer_dir)
from dmad_b200.models.h3 import H3Config, H3Model

safetensors = pytest.importorskip("safetensors.torch")


def _tiny_folder(tmp_path, shards=2):
    cfg = H3Config(dim=64, num_heads=2, ffn_dim=128, num_layers=2, refiner_layers=1, text_dim=64,
                   time_embed_dim=32)
    torch.manual_seed(0)
    src = H3Model(cfg)
    tf = tmp_path / "transformer"
    tf.mkdir()
    json.dump({"_class_name": "MiniMaxH3Transformer3DModel", "num_attention_heads": 2, "attention_head_dim": 32,
               "ffn_dim": 128, "num_layers": 2, "num_refiner_layers": 1, "text_embed_dim": 64, "time_embed_dim": 32,
               "in_channels": cfg.in_channels, "audio_in_channels": cfg.audio_in_channels,
               "patch_size": list(cfg.patch_size)}, open(tf / "config.json", "w"))
    sd = {k: v.contiguous() for k, v in src.state_dict().items()}
    keys = sorted(sd)
    wm = {}
    for i in range(shards):
        name = f"diffusion_pytorch_model-{i + 1:05d}-of-{shards:05d}.safetensors"
        part = {k: sd[k] for k in keys[i::shards]}
        safetensors.save_file(part, str(tf / name))
        wm.update({k: name for k in part})
    json.dump({"weight_map": wm}, open(tf / "diffusion_pytorch_model.safetensors.index.json", "w"))
    return cfg, src


def test_resolve_and_config(tmp_path):
    cfg, _ = _tiny_folder(tmp_path)
    assert resolve_transformer_dir(tmp_path) == tmp_path / "transformer"
    assert resolve_transformer_dir(tmp_path / "transformer") == tmp_path / "transformer"
    got = config_from_transformer_dir(tmp_path)
    assert (got.dim, got.num_heads, got.ffn_dim, got.num_layers, got.refiner_layers) == (64, 2, 128, 2, 1)
    with pytest.raises(FileNotFoundError):
        resolve_transformer_dir(tmp_path / "nothing")
    json.dump({"_class_name": "Other"}, open(tmp_path / "transformer" / "config.json", "w"))
    with pytest.raises(ValueError):
        resolve_transformer_dir(tmp_path)


def test_weights_roundtrip(tmp_path):
    cfg, src = _tiny_folder(tmp_path)
    dst = H3Model(H3Config(dim=64, num_heads=2, ffn_dim=128, num_layers=2, refiner_layers=1, text_dim=64,
                           time_embed_dim=32))
    missing, unexpected = load_transformer_weights(dst, tmp_path)
    assert not missing and not unexpected
    for k, v in src.state_dict().items():
        torch.testing.assert_close(dst.state_dict()[k], v, rtol=0, atol=0)


def test_strict_mismatch(tmp_path):
    _, src = _tiny_folder(tmp_path, shards=1)
    tf = tmp_path / "transformer"
    (tf / "diffusion_pytorch_model.safetensors.index.json").unlink()
    extra = {"not.a.param": torch.zeros(3)}
    safetensors.save_file(extra, str(tf / "zz_extra.safetensors"))
    with pytest.raises(KeyError):
        load_transformer_weights(H3Model(H3Config(dim=64, num_heads=2, ffn_dim=128, num_layers=2, refiner_layers=1,
                                                  text_dim=64, time_embed_dim=32)), tmp_path)
    model, (missing, unexpected) = load_transformer(tmp_path, dtype=torch.float32, strict=False)
    assert unexpected == ["not.a.param"] and not missing


def test_cli_loads_model_dir(tmp_path):
    """The CLI takes the network shape and weights from ``--model-dir`` (no text encoder or VAE weights)."""
    import os

    from dmad_b200.cli.h3_inference import main

    _tiny_folder(tmp_path)
    (tmp_path / "vae").mkdir()
    json.dump({"spatial_downsample_factors": [2, 2, 2, 2]}, open(tmp_path / "vae" / "config.json", "w"))
    (tmp_path / "p.txt").write_text("a fox\n", encoding="utf-8")
    main(["--model-dir", str(tmp_path), "--prompt-file", str(tmp_path / "p.txt"), "--output-dir",
          str(tmp_path / "out"), "--steps", "1", "--height", "64", "--width", "64", "--num-frames", "22",
          "--text-tokens", "4"])
    assert os.listdir(tmp_path / "out")


@pytest.mark.parametrize("extra", [["--low-vram", "24", "--chunk-rows", "40"],
                                   ["--low-vram", "8", "--weights-in-ram"]])
def test_cli_low_vram_streams_from_model_dir(tmp_path, extra):
    """--low-vram with a model folder: blocks stream from the shards (or a RAM copy), rows chunked;
    the latents equal the resident run's up to chunking round-off."""
    from dmad_b200.cli.h3_inference import main

    _tiny_folder(tmp_path)
    (tmp_path / "vae").mkdir()
    json.dump({"spatial_downsample_factors": [2, 2, 2, 2]}, open(tmp_path / "vae" / "config.json", "w"))
    args = ["--model-dir", str(tmp_path), "--prompt", "a fox", "--steps", "2", "--height", "64", "--width", "64",
            "--num-frames", "22", "--text-tokens", "4"]
    ref = main(args + ["--output-dir", str(tmp_path / "ref")])
    out = main(args + ["--output-dir", str(tmp_path / "low")] + extra)
    for (v, a), (rv, ra) in zip(out, ref):
        torch.testing.assert_close(v.float(), rv.float(), rtol=0.05, atol=0.05)
        torch.testing.assert_close(a.float(), ra.float(), rtol=0.05, atol=0.05)


def test_h3_dmad_trainer_starts_from_model_dir(tmp_path):
    """``model_dir`` in the H3 DMAD config: the student and the critic start from the folder's weights."""
    from dmad_b200.distill.h3_dmad import H3DMAD, H3DMADConfig

    cfg, src = _tiny_folder(tmp_path)
    hc = H3DMADConfig(height=64, width=64, num_frames=22, student_lora_rank=4, text_tokens=4,
                      model_dir=str(tmp_path))
    m = H3DMAD(hc, "cpu", dtype=torch.float32)
    assert m.cfg.model.dim == 64 and len(m.student.transformer_blocks) == 2
    want = src.state_dict()
    for net in (m.student, m.fake):
        got = net.state_dict()
        for k in ("proj_in.weight", "transformer_blocks.1.attn.to_k.weight", "transformer_blocks.0.ff.net.2.bias"):
            torch.testing.assert_close(got[k], want[k], rtol=0, atol=0)
    out = m.train_iteration()
    assert all(torch.isfinite(torch.tensor(v)) for v in out["student"].values())


def test_diffusers_pipeline_runner_matches_euler_inference(tmp_path):
    """The Diffusers-runner CLI (the reference's run_diffusers_pipeline.py flags) samples with the LoRA
    attached and the Euler step rule: the same latents as ``h3_inference --euler`` with the same settings,
    and one output per prompt."""
    import os

    from dmad_b200.cli.diffusers_pipeline import main as runner
    from dmad_b200.cli.h3_inference import main as h3
    from dmad_b200.lora import save_lora_file

    _tiny_folder(tmp_path)
    (tmp_path / "vae").mkdir()
    json.dump({"spatial_downsample_factors": [2, 2, 2, 2]}, open(tmp_path / "vae" / "config.json", "w"))
    g = torch.Generator().manual_seed(4)
    pairs = {f"transformer_blocks.{i}.attn.{n}": {"A": torch.randn(4, 64, generator=g) * 0.05,
                                                   "B": torch.randn(64, 4, generator=g) * 0.05}
             for i in range(2) for n in ("to_q", "to_v")}
    lora = str(tmp_path / "student.safetensors")
    save_lora_file(lora, pairs, 4, 4.0)
    common = ["--model-dir", str(tmp_path), "--lora", lora, "--prompt", "a fox", "--prompt", "a cat", "--steps", "2",
              "--height", "64", "--width", "64", "--num-frames", "22", "--text-tokens", "4", "--seed", "7"]
    out = runner(common + ["--output-dir", str(tmp_path / "runner")])
    ref = h3(common + ["--output-dir", str(tmp_path / "ref"), "--euler"])
    assert len(out) == 2
    for (v, a), (rv, ra) in zip(out, ref):
        assert torch.equal(v, rv) and torch.equal(a, ra)
    files = sorted(os.listdir(tmp_path / "runner"))
    assert "settings.json" in files and "0000.txt" in files and "0001.txt" in files
