"""Causal modes of the Wan network on CPU: a block-causal forward of the whole sequence equals the
chunk-by-chunk forward against the KV cache (append mode, RoPE at the chunk's frame offset); causal
sampling with a single chunk equals bidirectional sampling; KVCache bookkeeping (parity:
train/wan/rcm/utils/kv_cache.py, sample_videos.py:259-370)."""
import pytest
import torch


def _model():
    from dmad_b200.models.wan import WanConfig, WanModel

    torch.manual_seed(0)
    m = WanModel(WanConfig(dim=128, ffn_dim=256, num_heads=2, num_layers=2, text_dim=32, freq_dim=64))
    torch.nn.init.normal_(m.head.head.weight, std=0.05)
    return m.eval()


@pytest.mark.parametrize("first,chunk,local,sink", [(1, 2, 0, 0), (1, 1, 2, 1), (2, 1, 0, 0)])
def test_block_causal_forward_equals_cached_chunks(first, chunk, local, sink):
    from dmad_b200.models.kv_cache import CausalInferenceState, KVCacheMode
    from dmad_b200.ops.block_attention import AttnMaskSpec, BlockPattern

    m = _model()
    g = torch.Generator().manual_seed(1)
    T = first + 2 * chunk
    x = torch.randn(1, 16, T, 4, 8, generator=g)
    t = torch.rand(1, 1, generator=g)
    ctx = torch.randn(1, 6, 32, generator=g)
    ft = (4 // 2) * (8 // 2)
    pat = BlockPattern(ft, first, chunk)
    with torch.no_grad():
        full = m(x, t, ctx, attn_meta=AttnMaskSpec("block_causal", pat, local, sink))
        st = CausalInferenceState(len(m.blocks), T * ft, pat, local, sink, mode=KVCacheMode.APPEND)
        parts, f0, b = [], 0, 0
        while f0 < T:
            f1 = f0 + pat.block_frames(b)
            st.block_idx = b
            parts.append(m(x[:, :, f0:f1], t, ctx, inference_state=st))
            f0, b = f1, b + 1
    torch.testing.assert_close(torch.cat(parts, dim=2), full, rtol=1e-4, atol=1e-5)


def test_single_chunk_causal_sampling_equals_bidirectional():
    from dmad_b200.cli.wan_sample import sample_bidirectional
    from dmad_b200.samplers.causal import sample_causal

    m = _model()
    noise = torch.randn(1, 16, 3, 4, 8, generator=torch.Generator().manual_seed(2))
    ctx = torch.randn(1, 6, 32, generator=torch.Generator().manual_seed(3))
    steps = [0.9, 0.5, 0.0]
    a = sample_bidirectional(m, noise, steps, ctx, generator=torch.Generator().manual_seed(4))
    b = sample_causal(m, noise, steps, ctx, first_chunk_frames=3, chunk_frames=1,
                      generator=torch.Generator().manual_seed(4))
    torch.testing.assert_close(b, a, rtol=1e-5, atol=1e-5)
    c = sample_causal(m, noise, steps, ctx, first_chunk_frames=1, chunk_frames=1, unctx=torch.zeros_like(ctx),
                      guidance=3.0, context_from_last_step=True, generator=torch.Generator().manual_seed(4))
    assert c.shape == noise.shape and torch.isfinite(c).all()


def test_kv_cache_bookkeeping():
    from dmad_b200.models.kv_cache import KVCache

    c = KVCache(10)
    k = torch.arange(2 * 3 * 1 * 2, dtype=torch.float32).view(2, 3, 1, 2)
    assert c.append(k, -k) == (0, 3) and c.append(k + 100, -k) == (3, 6)
    assert c.get(0) == (None, None) and c.get(1)[0].shape[1] == 3 and c.get()[0].shape[1] == 6
    kk, _ = c.write_transient(k + 7, k, at=3)
    assert kk.shape[1] == 6 and c.current_len == 6 and torch.equal(kk[:, 3:], k + 7)
    c.compact_(torch.tensor([0, 4]))
    assert c.current_len == 2 and torch.equal(c.k[:, 1], (k + 7)[:, 1])
    with pytest.raises(RuntimeError):
        c.append(torch.zeros(2, 9, 1, 2), torch.zeros(2, 9, 1, 2))
    with pytest.raises(IndexError):
        c.get(3)
