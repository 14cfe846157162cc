"""CPU oracle: the reference's own Wan network (installed under baseline/_ref from the reference source)
with random weights, loaded into this package's WanModel through the shared state-dict layout, gives the
same output in fp32 -- uniform and per-frame timesteps (skipped when the reference is not installed)."""
import os
import sys

import pytest
import torch

REF = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "baseline", "_ref")


@pytest.fixture(scope="module")
def ref_wan():
    if not os.path.isdir(os.path.join(REF, "rcm")):
        pytest.skip("reference not installed")
    sys.path.insert(0, REF)
    try:
        import rcm.utils.rope as ref_rope
        from rcm.networks.wan2pt1 import WanModel
    except Exception as e:  # pragma: no cover - depends on the installed reference
        pytest.skip(f"reference Wan network does not import here: {e}")
    # the reference rotates with flash-attn's GPU kernel when that package imports; on CPU it must take
    # its own PyTorch fallback (rope.py:65-70)
    ref_rope.flash_apply_rotary_emb = None
    # and its SDPA backend list has no CPU entry (attention.py:72-116): give it the math backend
    import rcm.utils.attention as ref_attn
    from torch.nn.attention import SDPBackend, sdpa_kernel
    ref_attn._get_sdpa_config = lambda device, is_half: (0, [SDPBackend.MATH], sdpa_kernel)
    return WanModel


@pytest.mark.parametrize("per_frame", [False, True])
def test_wan_forward_matches_reference(ref_wan, per_frame):
    from dmad_b200.models.wan import WanConfig, WanModel

    torch.manual_seed(0)
    ref = ref_wan(dim=128, ffn_dim=256, freq_dim=64, text_dim=32, num_heads=2, num_layers=2, text_len=8).float()
    with torch.no_grad():
        for n, p in ref.named_parameters():  # the reference zero-initialises its head; make every part count
            p.add_(torch.randn_like(p) * 0.05)
    ref.eval()
    ours = WanModel(WanConfig(dim=128, ffn_dim=256, num_heads=2, num_layers=2, text_dim=32, freq_dim=64)).float()
    missing, unexpected = ours.load_state_dict(ref.state_dict(), strict=False)
    assert not [k for k in missing if not k.endswith(("_u", "_sn_gain"))], missing
    assert not unexpected, unexpected
    ours.eval()
    g = torch.Generator().manual_seed(1)
    x = torch.randn(1, 16, 3, 4, 8, generator=g)
    t = (torch.rand(1, 3, generator=g) if per_frame else torch.rand(1, 1, generator=g)) * 1000
    ctx = torch.randn(1, 8, 32, generator=g)
    with torch.no_grad():
        r = ref(x, t, ctx).float()
        o = ours(x, t, ctx).float()
    assert r.shape == o.shape
    torch.testing.assert_close(o, r, rtol=2e-4, atol=2e-4)
