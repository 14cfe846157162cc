"""The Qwen3-VL prompt conditioner on a tiny random Qwen3-VL: the truncated run (layers above the one
read skipped, final norm bypassed) equals ``hidden_states[layer]`` of the full model, the reference's
read-out (dmad_h3/text_encoder.py:51-66)."""
import pytest
import torch

transformers = pytest.importorskip("transformers")


def _tiny():
    from transformers import Qwen3VLConfig, Qwen3VLForConditionalGeneration

    cfg = Qwen3VLConfig(
        text_config=dict(vocab_size=300, hidden_size=64, intermediate_size=128, num_hidden_layers=4,
                         num_attention_heads=4, num_key_value_heads=2, head_dim=16,
                         rope_scaling={"rope_type": "default", "mrope_section": [2, 3, 3], "mrope_interleaved": True}),
        vision_config=dict(depth=1, hidden_size=32, intermediate_size=64, num_heads=2, out_hidden_size=64,
                           deepstack_visual_indexes=[0]))
    torch.manual_seed(0)
    return Qwen3VLForConditionalGeneration(cfg).eval()


class _Tok:
    def __call__(self, text, add_special_tokens=False):
        return {"input_ids": [3 + (ord(c) % 250) for c in text]}


@pytest.mark.parametrize("layer", [1, 2, 4])
def test_conditioner_reads_hidden_layer(layer):
    from dmad_b200.inference.text_encoder import Qwen3VLConditioner

    m = _tiny()
    cond = Qwen3VLConditioner(m, _Tok(), layer=layer, output_dtype=torch.float32)
    out = cond.encode("a red fox runs")
    ids = torch.tensor([_Tok()("a red fox runs")["input_ids"]])
    with torch.no_grad():
        ref = m.model(input_ids=ids, attention_mask=torch.ones_like(ids), mm_token_type_ids=torch.zeros_like(ids),
                      use_cache=False, output_hidden_states=True).hidden_states[layer]
    assert out["prompt_embeds"].shape == (1, ids.shape[1], 64)
    torch.testing.assert_close(out["prompt_embeds"], ref.float(), rtol=1e-5, atol=1e-5)
    assert out["text_token_tags"].tolist() == [1] * ids.shape[1]
    assert len(m.model.language_model.layers) == 4  # restored after the truncated run


def test_drop_unused_layers_and_read_prompts(tmp_path):
    from dmad_b200.inference.text_encoder import Qwen3VLConditioner, read_prompts

    m = _tiny()
    ids = torch.tensor([_Tok()("two cats")["input_ids"]])
    with torch.no_grad():
        ref = m.model(input_ids=ids, attention_mask=torch.ones_like(ids), mm_token_type_ids=torch.zeros_like(ids),
                      use_cache=False, output_hidden_states=True).hidden_states[2]
    cond = Qwen3VLConditioner(m, _Tok(), layer=2, drop_unused=True, output_dtype=torch.float32)
    assert len(m.model.language_model.layers) == 2
    torch.testing.assert_close(cond.encode("two cats")["prompt_embeds"], ref.float(), rtol=1e-5, atol=1e-5)
    (tmp_path / "p.txt").write_text("first\n\n second \n", encoding="utf-8")
    (tmp_path / "p.jsonl").write_text('{"prompt": "a"}\n{"prompt": "b"}\n', encoding="utf-8")
    assert read_prompts(tmp_path / "p.txt") == ["first", "second"]
    assert read_prompts(tmp_path / "p.jsonl") == ["a", "b"]


def test_prompt_cache_shards_and_merge(tmp_path):
    """encode-prompts over two shards then merge: the files the H3 pool reads, one condition per index."""
    from dmad_b200.data.h3_pool import data_file
    from dmad_b200.inference.text_encoder import Qwen3VLConditioner
    from dmad_b200.tools.h3_data import encode_prompts, merge_prompt_shards

    (tmp_path / "p.jsonl").write_text("".join(f'{{"prompt": "prompt number {i}"}}\n' for i in range(5)),
                                      encoding="utf-8")
    enc = Qwen3VLConditioner(_tiny(), _Tok(), layer=2)
    out = tmp_path / "cache"
    for r in range(2):
        encode_prompts(str(tmp_path / "p.jsonl"), str(out), enc, indices=[0, 2, 3, 4], shard=f"{r}/2")
    assert merge_prompt_shards(str(out)) == 4
    d = torch.load(data_file(str(out / "conditions"), "condition_00000003.pt"), weights_only=False)
    assert d["prompt"] == "prompt number 3" and d["source_index"] == 3
    pos = d["conditioning"]["positive"]
    assert pos["prompt_embeds"].shape[-1] == 64 and pos["prompt_embeds"].dtype == torch.bfloat16
    assert not (out / "conditions" / "condition_00000001.pt").exists()
