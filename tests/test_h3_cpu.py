"""H3 packing geometry, sampling rules, LoRA file round trip and the exact ComfyUI conversion."""
import os
import tempfile

import torch

from dmad_b200.inference.h3 import (H3Geometry, audio_latent_num_frames, build_packed_sequence, build_row_timesteps,
                                    latent_shape_of, shift_sigma, sigma_grid, video_latent_num_frames)


def test_frame_counts_and_shapes():
    assert video_latent_num_frames(124) == 37
    assert audio_latent_num_frames(124) == 207
    s = latent_shape_of(768, 1344, 124, H3Geometry())
    assert s["video_tokens"] == (1, 37 * 24 * 42, 96) and s["audio_tokens"] == (1, 414, 32)
    try:
        video_latent_num_frames(100)
        raise AssertionError("17n+5 check missing")
    except ValueError:
        pass


def test_packed_layout():
    lay = build_packed_sequence(torch.ones(5, dtype=torch.long), 7, 8, 8, 3)
    assert lay.sequence_length == 5 + 6 + 7 * 16
    assert lay.token_tags[:5].eq(1).all() and lay.token_tags[5:11].eq(2).all() and lay.token_tags[11:].eq(0).all()
    # audio rows: time continues after the text; the two channels sit at the first / last width position
    assert torch.equal(lay.position_ids[5:8, 0], torch.tensor([5.0, 6.0, 7.0], dtype=torch.float64))
    assert lay.position_ids[5, 2] < lay.position_ids[8, 2]
    # temporal grid pattern (1, 4, 4, 4, 4) x 5/3
    t = lay.position_ids[11::16, 0]
    d = (t[1:] - t[:-1]) * 3 / 5
    assert torch.allclose(d, torch.tensor([1.0, 4, 4, 4, 4, 1], dtype=torch.float64))
    ts, ti = build_row_timesteps(lay, torch.tensor(0.75), torch.tensor(0.5))
    assert ts.tolist() == [0.25, 0.5] and (ti[5:11] == 1).all() and (ti[:5] == 0).all()


def test_sigma_grid():
    g = sigma_grid(4, 12.0)
    assert g[0] == 1.0 and g[-1] == 0.0 and len(g) == 5
    assert torch.allclose(g[1], shift_sigma(torch.tensor(0.75), 12.0))


def test_lora_roundtrip_and_comfyui():
    from dmad_b200 import lora as L
    from dmad_b200.models.h3 import H3Config, H3Model
    from dmad_b200.tools.lora_comfyui import convert, verify
    torch.manual_seed(0)
    cfg = H3Config(dim=128, num_heads=1, ffn_dim=192, num_layers=2, refiner_layers=1, text_dim=32,
                   time_embed_dim=64)
    m = H3Model(cfg)
    m.enable_lora(4)
    for n, p in m.named_parameters():
        if "lora_B" in n:
            p.data.normal_(0, 0.1)
    pairs = L.lora_pairs_from_model(m)
    assert len(pairs) == 2 * 6
    with tempfile.TemporaryDirectory() as d:
        f = os.path.join(d, "x.safetensors")
        L.save_lora_file(f, pairs, 4, 4.0)
        p2, meta = L.read_lora_file(f)
        assert L.lora_rank_alpha(p2, meta) == (4, 4.0)
        for k in pairs:
            assert torch.equal(pairs[k]["A"], p2[k]["A"]) and torch.equal(pairs[k]["B"], p2[k]["B"])
        out = convert(p2, 4, 4.0)
        verify(p2, out)
        assert out["diffusion_model.blocks.0.attn.qkv_proj.lora_A.weight"].shape[0] == 12


def test_h3_dmad_iterations_cpu():
    from dmad_b200.distill.h3_dmad import H3DMAD, H3DMADConfig
    from dmad_b200.models.h3 import H3Config
    cfg = H3DMADConfig(model=H3Config(dim=64, num_heads=1, ffn_dim=96, num_layers=2, refiner_layers=1, text_dim=16,
                                      time_embed_dim=32), height=64, width=64, num_frames=22, student_lora_rank=4,
                       text_tokens=4)
    m = H3DMAD(cfg, "cpu", dtype=torch.float32)
    before = [p.detach().clone() for p in m.s_params]
    for _ in range(2):
        out = m.train_iteration()
        assert all(torch.isfinite(torch.tensor(v)) for v in out["student"].values())
    assert any(not torch.equal(a, b) for a, b in zip(before, m.s_params))
    sd = m.critic_state()
    m.load_critic_state(sd)
    assert m.student_steps == 2 and m.ema_banks[0].t == 2


def test_h3_checkpoint_exports_loras(tmp_path):
    """The training CLI on the H3 family writes the student / EMA / critic LoRA files into each checkpoint."""
    import os

    from dmad_b200.cli.train import main
    from dmad_b200.lora import read_lora_file

    cfg = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "configs", "h3_dmad.yaml")
    net = ("model.net={dim: 64, num_heads: 1, ffn_dim: 96, num_layers: 2, refiner_layers: 1, text_dim: 16, "
           "time_embed_dim: 32}")
    main(["--config", cfg, net, "model.distill.student_lora_rank=4", "model.distill.height=64",
          "model.distill.width=64", "model.distill.num_frames=22", "model.distill.text_tokens=6",
          "model.distill.gradient_checkpointing=false", f"training.output_dir={tmp_path}", "training.max_iters=1",
          "training.save_every=1"])
    ck = tmp_path / "checkpoint-000000001"
    for f in ("pytorch_lora_weights.safetensors", "ema_lora/pytorch_lora_weights.safetensors",
              "ema2_lora/pytorch_lora_weights.safetensors", "fake_lora/pytorch_lora_weights.safetensors"):
        assert (ck / f).exists(), f
    pairs, meta = read_lora_file(str(ck / "ema_lora" / "pytorch_lora_weights.safetensors"))
    assert pairs and meta.get("ema_gamma") == "6.94"
