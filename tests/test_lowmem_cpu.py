"""Low-VRAM streaming on a CPU device (the native engine in host mode: synchronous copies, the same
schedule): the streamed rollout equals the resident one, weights stream from byte ranges of the
safetensors shards or from an int8 cache directory checked against the shards' fingerprint, row-chunked
blocks match the full-width forward, and the streamed text encoder equals the resident conditioner
(parity: dmad_h3/lowmem.py, the --low-vram path)."""
import copy
import json
import os

import pytest
import torch

from dmad_b200.inference.h3 import (H3Geometry, build_packed_sequence, build_row_timesteps, latent_shape_of,
                                    load_transformer, rollout, sigma_grid)
from dmad_b200.inference.lowmem import LayerStreamer, LowMemH3, build_streamed_h3, chunked_block_forward
from dmad_b200.models.h3 import H3Config, H3Model

safetensors = pytest.importorskip("safetensors.torch")

CFG = dict(dim=256, num_heads=2, ffn_dim=512, num_layers=3, refiner_layers=1, text_dim=128, time_embed_dim=128)


def _model():
    torch.manual_seed(0)
    m = H3Model(H3Config(**CFG))
    for p in m.parameters():
        p.data.normal_(0, 0.03)
    return m.eval().requires_grad_(False)


def _save(m, tmp_path):
    tf = tmp_path / "transformer"
    tf.mkdir(exist_ok=True)
    c = CFG
    json.dump({"_class_name": "MiniMaxH3Transformer3DModel", "num_attention_heads": c["num_heads"],
               "attention_head_dim": c["dim"] // c["num_heads"], "ffn_dim": c["ffn_dim"], "num_layers": c["num_layers"],
               "num_refiner_layers": c["refiner_layers"], "text_embed_dim": c["text_dim"],
               "time_embed_dim": c["time_embed_dim"]}, open(tf / "config.json", "w"))
    sd = {k: v.contiguous() for k, v in m.state_dict().items()}
    keys = sorted(sd)
    safetensors.save_file({k: sd[k] for k in keys[::2]}, str(tf / "part-1.safetensors"))
    safetensors.save_file({k: sd[k] for k in keys[1::2]}, str(tf / "part-2.safetensors"))
    return tf


def _case(steps=2):
    geo = H3Geometry()
    shape = latent_shape_of(64, 64, 22, geo)
    lay = build_packed_sequence(torch.ones(12, dtype=torch.long), shape["latent_frames"], shape["latent_height"],
                                shape["latent_width"], shape["audio_latents"])
    vs, as_ = sigma_grid(steps, 12.0), sigma_grid(steps, 2.0)
    ts = [build_row_timesteps(lay, vs[s], as_[s])[0] for s in range(steps)]
    pe = torch.randn(1, 12, CFG["text_dim"], generator=torch.Generator().manual_seed(3))
    return geo, shape, lay, vs, as_, ts, pe


def _run(model, case, lm=None):
    geo, shape, lay, vs, as_, ts, pe = case
    kw = {}
    if lm is not None:
        if not lm._text_cache:
            lm.precompute_text([pe])
        kw = dict(text_features=lm.text_features(pe), adaln_tables_per_step=lm.tables)
    return rollout(model, pe, lay, shape, geo, vs, as_, 7, torch.device("cpu"), **kw)


def test_streamed_in_memory_equals_resident():
    m = _model()
    case = _case()
    ref = _run(copy.deepcopy(m), case)
    lm = LowMemH3(copy.deepcopy(m), "cpu", case[5])
    out = _run(lm.model, case, lm)
    lm.close()
    assert torch.equal(out[0], ref[0]) and torch.equal(out[1], ref[1])


@pytest.mark.parametrize("in_ram", [False, True])
def test_streamed_from_shards_equals_resident(tmp_path, in_ram):
    m = _model()
    _save(m, tmp_path)
    case = _case()
    ref = _run(load_transformer(tmp_path, dtype=torch.float32), case)
    model, source = build_streamed_h3(tmp_path, "cpu", dtype=torch.float32)
    assert model.transformer_blocks[0].attn.qkv.weight.device.type == "meta"
    lm = LowMemH3(model, "cpu", case[5], source=source, cache_in_ram=in_ram)
    assert (lm.streamer.host is None) == (not in_ram)
    out = _run(lm.model, case, lm)
    out2 = _run(lm.model, case, lm)  # a second pass re-reads the shards through the staging buffers
    st = lm.streamer.stats()
    lm.close()
    # every block evaluation copied one block's layout; read from the shards when not cached in RAM
    assert st["copies"] >= 2 * 2 * CFG["num_layers"]
    assert (st["bytes_read_from_files"] > 0) == (not in_ram)
    assert torch.equal(out[0], ref[0]) and torch.equal(out[1], ref[1])
    assert torch.equal(out2[0], ref[0])


def test_int8_disk_cache_manifest(tmp_path):
    m = _model()
    _save(m, tmp_path)
    case = _case()
    ref = _run(load_transformer(tmp_path, dtype=torch.float32), case)
    cache = tmp_path / "cache"
    model, source = build_streamed_h3(tmp_path, "cpu", dtype=torch.float32)
    with pytest.raises(ValueError):
        LowMemH3(copy.deepcopy(model), "cpu", case[5], codec="int8", source=source, cache_in_ram=False)
    lm = LowMemH3(model, "cpu", case[5], codec="int8", source=source, cache_in_ram=False, cache_dir=cache)
    assert any(it.int8 for lay in lm.streamer.layouts for it in lay.params)
    out = _run(lm.model, case, lm)
    lm.close()
    rel = (out[0] - ref[0]).norm() / ref[0].norm()
    assert 0 < rel < 0.05  # quantised weights: close, not equal
    index = json.load(open(cache / "index.json"))
    assert len(index["blocks"]) == CFG["num_layers"] and len(index["source"]) == 2
    stamp = {f: os.stat(cache / f).st_mtime_ns for f in os.listdir(cache)}
    model, source = build_streamed_h3(tmp_path, "cpu", dtype=torch.float32)
    lm = LowMemH3(model, "cpu", case[5], codec="int8", source=source, cache_in_ram=False, cache_dir=cache)
    out2 = _run(lm.model, case, lm)
    lm.close()
    assert {f: os.stat(cache / f).st_mtime_ns for f in os.listdir(cache)} == stamp  # reused, not rewritten
    assert torch.equal(out2[0], out[0])


def test_chunked_block_forward_matches():
    m = _model()
    case = _case(1)
    ref = _run(copy.deepcopy(m), case)
    mc = copy.deepcopy(m)
    for b in mc.transformer_blocks:
        b.forward = chunked_block_forward(b, 37)  # several uneven chunks
    out = _run(mc, case)
    torch.testing.assert_close(out[0], ref[0], rtol=1e-4, atol=1e-5)
    torch.testing.assert_close(out[1], ref[1], rtol=1e-4, atol=1e-5)


def test_lora_on_streamed_model(tmp_path):
    from dmad_b200.lora import attach_lora

    m = _model()
    _save(m, tmp_path)
    case = _case(1)
    g = torch.Generator().manual_seed(5)
    pairs = {f"transformer_blocks.{i}.attn.{n}": {"A": torch.randn(4, 256, generator=g) * 0.05,
                                                   "B": torch.randn(256, 4, generator=g) * 0.05}
             for i in range(CFG["num_layers"]) for n in ("to_q", "to_v")}
    ref_m = load_transformer(tmp_path, dtype=torch.float32)
    attach_lora(ref_m, pairs, 4, 4.0)
    ref = _run(ref_m, case)
    model, source = build_streamed_h3(tmp_path, "cpu", dtype=torch.float32)
    attach_lora(model, pairs, 4, 4.0)
    lm = LowMemH3(model, "cpu", case[5], source=source, cache_in_ram=False, chunk_rows=50)
    out = _run(lm.model, case, lm)
    lm.close()
    torch.testing.assert_close(out[0], ref[0], rtol=1e-4, atol=1e-5)


def test_streamer_rejects_unloaded_parameters():
    with torch.device("meta"):
        m = H3Model(H3Config(**CFG))
    with pytest.raises(ValueError):
        LayerStreamer(list(m.transformer_blocks), "cpu")


transformers = pytest.importorskip("transformers")


class _Tok:
    def __call__(self, text, add_special_tokens=False):
        return {"input_ids": [3 + (ord(c) % 250) for c in text]}


def test_streamed_text_encoder_equals_conditioner(tmp_path):
    from transformers import Qwen3VLConfig, Qwen3VLForConditionalGeneration

    from dmad_b200.inference.lowmem import LowMemTextEncoder
    from dmad_b200.inference.text_encoder import Qwen3VLConditioner

    cfg = Qwen3VLConfig(
        text_config=dict(vocab_size=300, hidden_size=64, intermediate_size=128, num_hidden_layers=4,
                         num_attention_heads=4, num_key_value_heads=2, head_dim=16,
                         rope_scaling={"rope_type": "default", "mrope_section": [2, 3, 3], "mrope_interleaved": True}),
        vision_config=dict(depth=1, hidden_size=32, intermediate_size=64, num_heads=2, out_hidden_size=64,
                           deepstack_visual_indexes=[0]))
    torch.manual_seed(0)
    full = Qwen3VLForConditionalGeneration(cfg).eval()
    full.save_pretrained(str(tmp_path / "text_encoder"), safe_serialization=True)
    ref = Qwen3VLConditioner(full, _Tok(), layer=3, output_dtype=torch.float32).encode("a red fox runs")
    enc = LowMemTextEncoder(tmp_path, "cpu", layer=3, dtype=torch.float32, tokenizer=_Tok())
    assert len(enc.lm.layers) == 3
    out = enc.encode("a red fox runs", output_dtype=torch.float32)
    out2 = enc.encode("a red fox runs", output_dtype=torch.float32)
    enc.close()
    torch.testing.assert_close(out["prompt_embeds"], ref["prompt_embeds"], rtol=1e-5, atol=1e-5)
    assert torch.equal(out2["prompt_embeds"], out["prompt_embeds"])
    assert out["text_token_tags"].tolist() == ref["text_token_tags"].tolist()
