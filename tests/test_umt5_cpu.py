"""umT5 encoder on CPU: T5 relative buckets (exact / logarithmic / sign halves), the XXL parameter
count and key layout, padding rows zeroed, and padding not changing the encoding of real tokens."""
import torch


def test_relative_buckets():
    from dmad_b200.models.umt5 import relative_bucket

    rel = torch.tensor([-200, -64, -9, -8, -7, -1, 0, 1, 7, 8, 9, 64, 200])
    b = relative_bucket(rel, 32, 128).tolist()
    assert b[6] == 0 and b[5] == 1 and b[7] == 17         # exact region, sign in the upper half
    assert b[4] == 7 and b[8] == 23
    assert b[3] >= 8 and b[9] >= 24                      # logarithmic beyond 8
    assert b[0] == 15 and b[-1] == 31                    # clamped at the last bucket of each half
    assert b[1] <= b[0] and b[11] <= b[12]


def test_xxl_size_and_keys():
    from dmad_b200.models.umt5 import UMT5Encoder

    with torch.device("meta"):
        m = UMT5Encoder()
    n = sum(p.numel() for p in m.parameters())
    assert 5.5e9 < n < 5.8e9, n
    keys = set(m.state_dict())
    for k in ("token_embedding.weight", "blocks.0.attn.q.weight", "blocks.23.ffn.gate.0.weight",
              "blocks.5.ffn.fc1.weight", "blocks.5.pos_embedding.embedding.weight", "norm.weight"):
        assert k in keys


def test_encode_masks_padding():
    from dmad_b200.models.umt5 import TextEncoder, UMT5Config

    torch.manual_seed(0)
    cfg = UMT5Config(vocab=1000, dim=64, dim_attn=64, dim_ffn=128, num_heads=4, num_layers=2, text_len=16)
    te = TextEncoder(cfg, dtype=torch.float32)
    ctx = te.encode(["a red fox jumps", "the quick brown fox jumps over the lazy dog today"])
    assert ctx.shape == (2, 16, 64)
    assert ctx[0, 5:].abs().max() == 0 and ctx[0, :5].abs().max() > 0      # 4 words + EOS
    short = te.encode(["a red fox jumps"])
    assert torch.allclose(short[0], ctx[0], atol=1e-5)
