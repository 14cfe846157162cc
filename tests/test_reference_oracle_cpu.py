"""CPU oracles: the reference's own modules (installed under baseline/_ref from the reference source) with
random weights, loaded into this package's modules through the shared state-dict layouts, give the same
outputs in fp32 -- the Wan DiT (uniform and per-frame timesteps), the causal video VAE (encode and decode),
the umT5 encoder with padding -- and the reference's block-mask predicates equal this package's key-range
rectangles.  The reference comes from baseline/_ref or the reference checkout; the tests fail when
neither is present (tests/_reference_src.py)."""
import os
import sys

import pytest
import torch

from _reference_src import wan_tree


def _stub_io_deps():
    """Stand-ins for packages the reference imports only for video IO, text cleaning and log colours."""
    import types

    if "imageio" not in sys.modules:
        try:
            import imageio  # noqa: F401
        except ImportError:
            pkg = types.ModuleType("imageio")
            pkg.__path__ = []
            sys.modules["imageio"] = pkg
            sys.modules["imageio.v3"] = types.ModuleType("imageio.v3")
    for name, attr in (("ftfy", "fix_text"), ("termcolor", "colored")):
        try:
            __import__(name)
        except ImportError:
            mod = types.ModuleType(name)
            setattr(mod, attr, lambda text, *a, **k: text)
            sys.modules[name] = mod


@pytest.fixture(scope="module")
def ref_wan():
    REF = wan_tree()
    if REF not in sys.path:
        sys.path.insert(0, REF)
    try:
        import rcm.utils.rope as ref_rope
        from rcm.networks.wan2pt1 import WanModel
    except Exception as e:  # pragma: no cover - depends on the installed reference
        pytest.fail(f"reference Wan network does not import: {e}")
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


def test_wan_vae_matches_reference():
    """The reference's chunked causal VAE (first frame, then 4-frame chunks with feature caches; one
    latent frame at a time when decoding) against this package's whole-clip causal VAE, same weights."""
    REF = wan_tree()
    if REF not in sys.path:
        sys.path.insert(0, REF)
    _stub_io_deps()
    try:
        from rcm.tokenizers.wan2pt1 import WanVAE_
    except Exception as e:  # pragma: no cover
        pytest.fail(f"reference VAE does not import: {e}")
    from dmad_b200.models.wan_vae import WanVAEModel

    torch.manual_seed(0)
    ref = WanVAE_(dim=16, z_dim=4, dim_mult=[1, 2, 4, 4], num_res_blocks=1, attn_scales=[],
                  temperal_downsample=[False, True, True]).eval()
    with torch.no_grad():
        for p in ref.parameters():
            p.add_(torch.randn_like(p) * 0.02)
    ours = WanVAEModel(dim=16, z_dim=4, dim_mult=(1, 2, 4, 4), num_res_blocks=1,
                       temporal_downsample=(False, True, True)).eval()
    ours.load_state_dict(ref.state_dict())
    g = torch.Generator().manual_seed(2)
    x = torch.randn(1, 3, 9, 32, 32, generator=g)
    z = torch.randn(1, 4, 3, 4, 4, generator=g)
    scale = [torch.zeros(4), torch.ones(4)]
    with torch.no_grad():
        mu_ref = ref.encode(x, scale)
        mu = ours.conv1(ours.encoder(x))[:, :4]
        dec_ref = ref.decode(z, scale)
        dec = ours.decoder(ours.conv2(z))
    torch.testing.assert_close(mu, mu_ref, rtol=1e-4, atol=1e-4)
    torch.testing.assert_close(dec, dec_ref, rtol=1e-4, atol=1e-4)


def test_umt5_encoder_matches_reference():
    """The reference's umT5 encoder (per-layer relative position buckets, shared_pos=False as umT5 uses)
    against this package's encoder with the same weights, with a padding mask."""
    REF = wan_tree()
    if REF not in sys.path:
        sys.path.insert(0, REF)
    _stub_io_deps()
    saved = torch.cuda.current_device
    torch.cuda.current_device = lambda: 0  # a default argument of the reference's encoder wrapper (umt5.py:485)
    try:
        from rcm.utils.umt5 import T5Encoder
    except Exception as e:  # pragma: no cover
        pytest.fail(f"reference umT5 does not import: {e}")
    finally:
        torch.cuda.current_device = saved
    from dmad_b200.models.umt5 import UMT5Config, UMT5Encoder

    torch.manual_seed(0)
    ref = T5Encoder(vocab=300, dim=64, dim_attn=64, dim_ffn=128, num_heads=4, num_layers=2, num_buckets=32,
                    shared_pos=False, dropout=0.0).eval()
    ours = UMT5Encoder(UMT5Config(vocab=300, dim=64, dim_attn=64, dim_ffn=128, num_heads=4, num_layers=2,
                                  num_buckets=32, text_len=16)).eval()
    missing, unexpected = ours.load_state_dict(ref.state_dict(), strict=False)
    assert not missing and not unexpected, (missing, unexpected)
    ids = torch.randint(1, 300, (2, 16), generator=torch.Generator().manual_seed(3))
    mask = torch.ones(2, 16, dtype=torch.long)
    mask[1, 11:] = 0
    with torch.no_grad():
        r = ref(ids, mask)
        o = ours(ids, mask)
    torch.testing.assert_close(o, r, rtol=1e-4, atol=1e-4)


def test_block_masks_match_reference_predicate():
    """Key-range rectangles of ``mask_ranges`` against the reference's own mask functions
    (blockmask.py ``_make_mask_fn``) for block-causal (windows, sinks, query offsets) and teacher forcing."""
    import itertools

    REF = wan_tree()
    if REF not in sys.path:
        sys.path.insert(0, REF)
    try:
        from rcm.utils import blockmask as rb
    except Exception as e:  # pragma: no cover
        pytest.skip(f"reference block masks do not import here: {e}")
    from dmad_b200.ops.block_attention import AttnMaskSpec, BlockPattern, mask_ranges

    layer = rb.FlexOrSdpaLocalAttention.__new__(rb.FlexOrSdpaLocalAttention)  # only _make_mask_fn is used
    n = 0
    for ft, fc, cf, local, sink in itertools.product((3, 4), (1, 2), (1, 2), (0, 1, 2, 3), (0, 1, 2)):
        cases = []
        for qbo in (0, 1, 2):
            pre = BlockPattern(ft, fc, cf).blocks_to_tokens(qbo)
            Q = BlockPattern(ft, fc, cf).blocks_to_tokens(qbo + 3) - pre
            cases.append(("block_causal", dict(q_block_offset=qbo), Q, pre + Q))
        for clean in (2, 3):
            L = 2 * BlockPattern(ft, fc, cf).blocks_to_tokens(clean)
            cases.append(("teacher_forcing", dict(clean_blocks=clean), L, L))
        for mode, extra, Q, KV in cases:
            ref_spec = rb.AttnMaskSpec(mode=mode, pattern=rb.BlockPattern(ft, fc, cf), local_attn_blocks=local,
                                       sink_blocks=sink, **extra)
            fn, _ = layer._make_mask_fn(ref_spec, Q, KV)
            qi = torch.arange(Q)[:, None]
            ki = torch.arange(KV)[None, :]
            ref = fn(0, 0, qi, ki).expand(Q, KV)
            ours = torch.zeros(Q, KV, dtype=torch.bool)
            spec = AttnMaskSpec(mode, BlockPattern(ft, fc, cf), local, sink, **extra)
            for q0, q1, rng in mask_ranges(spec, Q, KV):
                for a, b in rng:
                    ours[q0:q1, a:b] = True
            assert torch.equal(ours, ref), (mode, ft, fc, cf, local, sink, extra)
            n += 1
    assert n > 200


def test_kv_cache_matches_reference():
    """The same sequence of cache operations on the reference's KVCache and this package's: appends,
    prefixes by chunk count, transient writes and compaction leave identical contents."""
    REF = wan_tree()
    if REF not in sys.path:
        sys.path.insert(0, REF)
    try:
        from rcm.utils.kv_cache import KVCache as RefKV
    except Exception as e:  # pragma: no cover
        pytest.fail(f"reference KV cache does not import: {e}")
    from dmad_b200.models.kv_cache import KVCache

    g = torch.Generator().manual_seed(0)
    mk = lambda n: torch.randn(2, n, 3, 4, generator=g)  # noqa: E731
    ref, ours = RefKV(20), KVCache(20)
    for n in (4, 6, 5):
        k, v = mk(n), mk(n)
        assert ref.append(k, v) == ours.append(k, v)
    for br in (None, 0, 1, 2, 3):
        a, b = ref.get(br), ours.get(br)
        assert (a[0] is None) == (b[0] is None)
        if a[0] is not None:
            assert torch.equal(a[0], b[0]) and torch.equal(a[1], b[1])
        assert ref.get_prefix_end(br) == ours.get_prefix_end(br)
    k, v = mk(3), mk(3)
    ra, oa = ref.write_transient(k, v, 10), ours.write_transient(k, v, 10)
    assert torch.equal(ra[0], oa[0]) and ref.current_len == ours.current_len
    keep = torch.tensor([0, 3, 7, 14])
    ref.compact_(keep)
    ours.compact_(keep)
    assert ref.current_len == ours.current_len
    assert torch.equal(ref.k[:, :ref.cur], ours.k[:, :ours.cur]) and torch.equal(ref.v[:, :ref.cur], ours.v[:, :ours.cur])


@pytest.mark.parametrize("kind,order,smax", [("euler", 1, 1.0), ("unipc", 2, 1.0), ("unipc", 3, 0.999)])
def test_teacher_samplers_match_reference(kind, order, smax):
    """Euler and UniPC (bh2) trajectories of a fixed velocity field through the reference's samplers and
    this package's, 20 shifted steps.  (Third order starts below sigma = 1: from sigma = 1 the log-SNR of
    the first step is infinite and the third-order corrector of the reference, like this one, is NaN.)"""
    REF = wan_tree()
    if REF not in sys.path:
        sys.path.insert(0, REF)
    try:
        from rcm.samplers.euler import FlowEulerSampler as RefEuler
        from rcm.samplers.unipc import FlowUniPCMultistepSampler as RefUniPC
    except Exception as e:  # pragma: no cover
        pytest.skip(f"reference samplers do not import here: {e}")
    from dmad_b200.samplers import FlowEulerSampler, FlowUniPCSampler

    if kind == "euler":
        ref, ours = RefEuler(sigma_max=smax), FlowEulerSampler(sigma_max=smax)
        ref.set_timesteps(20, shift=3.0, device="cpu")
    else:
        ref, ours = RefUniPC(solver_order=order, sigma_max=smax), FlowUniPCSampler(solver_order=order, sigma_max=smax)
        ref.set_timesteps(20, device="cpu", shift=3.0)
    ours.set_timesteps(20, shift=3.0, device="cpu")

    def vel(x, t):
        return -0.3 * x + 0.1 * torch.sin(t / 1000.0 * 3.0)

    x0 = torch.randn(2, 4, 6, generator=torch.Generator().manual_seed(0), dtype=torch.float64)
    xr, xo = x0.clone(), x0.clone()
    for t in ref.timesteps:
        xr = ref.step(vel(xr, t), t, xr)
    for t in ours.timesteps:
        xo = ours.step(vel(xo, t), t, xo)
    torch.testing.assert_close(xo.double(), xr.double(), rtol=1e-5, atol=2e-6)  # the reference runs in fp32


def test_lr_schedules_match_reference():
    """The Wan stack's LambdaLinear / LambdaWarmUpCosine multipliers (two cycles) against this package's."""
    REF = wan_tree()
    if REF not in sys.path:
        sys.path.insert(0, REF)
    try:
        from rcm.utils.lr_scheduler import LambdaLinearScheduler, LambdaWarmUpCosineScheduler
    except Exception as e:  # pragma: no cover
        pytest.skip(f"reference schedulers do not import here: {e}")
    from dmad_b200.runtime.lr import LAMBDA_LINEAR_DEFAULT, lambda_factor

    kw = dict(warm_up_steps=[10, 5], cycle_lengths=[50, 40], f_start=[0.01, 0.2], f_max=[1.0, 0.8], f_min=[0.1, 0.05])
    lin, cos = LambdaLinearScheduler(**kw), LambdaWarmUpCosineScheduler(**kw)
    for n in range(90):
        assert abs(lambda_factor(n, **kw) - lin(n)) < 1e-12, n
        assert abs(lambda_factor(n, cosine=True, **kw) - cos(n)) < 1e-12, n
    default = LambdaLinearScheduler(**LAMBDA_LINEAR_DEFAULT)
    for n in (0, 1, 50, 99, 100, 5000):
        assert abs(lambda_factor(n, **LAMBDA_LINEAR_DEFAULT) - default(n)) < 1e-12, n


def test_time_utilities_match_reference():
    """RF / TrigFlow time conversions, the log-normal and shifted-uniform samplers (same seed, same draws
    and inverse CDFs) and the rectified-flow TrigFlow scaling."""
    REF = wan_tree()
    if REF not in sys.path:
        sys.path.insert(0, REF)
    try:
        from rcm.utils import timestep_utils as rt
        from rcm.utils.denoiser_scaling import RectifiedFlow_TrigFlowWrapper
    except Exception as e:  # pragma: no cover
        pytest.skip(f"reference time utilities do not import here: {e}")
    from dmad_b200.algorithms import timesteps as ot

    t = torch.linspace(0.01, 0.99, 37, dtype=torch.float64)
    for name in ("rf_to_trig_time", "trig_to_rf_time", "sigma_to_rf_time", "rf_to_sigma"):
        torch.testing.assert_close(getattr(ot, name)(t), getattr(rt, name)(t))
    for s in (1.0, 3.0, 5.0):
        torch.testing.assert_close(ot.shift_rf_time(t, s), rt.shift_rf_time(t, s))
        torch.testing.assert_close(ot.inverse_shift_rf_time(t, s), rt.inverse_shift_rf_time(t, s))
    for ours, ref in ((ot.LogNormal(-0.8, 1.6), rt.LogNormal(-0.8, 1.6)), (ot.UniformShift(5.0), rt.UniformShift(5.0))):
        torch.manual_seed(3)
        a = ours((64, 1), device="cpu")
        torch.manual_seed(3)
        b = ref((64, 1), device="cpu")
        torch.testing.assert_close(a, b)
        torch.testing.assert_close(ours.icdf_rf(t), ref.icdf_rf(t))
        torch.testing.assert_close(ours.cdf_rf(t), ref.cdf_rf(t), rtol=1e-6, atol=1e-9)
    trig = ot.rf_to_trig_time(t)
    for a, b in zip(ot.TrigFlowScaling(t_scaling_factor=1000.0)(trig),
                    RectifiedFlow_TrigFlowWrapper(t_scaling_factor=1000.0)(trig)):
        torch.testing.assert_close(a, b)


def test_edm_unet_matches_reference():
    """The config-1 EDM U-Net against the reference's own EDMPrecond / DhariwalUNet
    (train/image/third_party/edm/training/networks.py), weights moved through the shared state dict:
    the denoised output and the critic's bottleneck features agree in fp32."""
    from _reference_src import image_tree

    from dmad_b200.models.edm import config1_unet

    tree = image_tree()
    for p in (tree, os.path.join(tree, "third_party", "edm")):
        if p not in sys.path:
            sys.path.insert(0, p)
    from third_party.edm.training.networks import EDMPrecond as RefPrecond

    torch.manual_seed(0)
    ref = RefPrecond(img_resolution=64, img_channels=3, label_dim=1000, use_fp16=False, sigma_min=0,
                     sigma_max=float("inf"), sigma_data=0.5, model_type="DhariwalUNet", augment_dim=0,
                     model_channels=64, channel_mult=[1, 2, 2], channel_mult_emb=4, num_blocks=1,
                     attn_resolutions=[16], dropout=0.0, label_dropout=0)
    del ref.model.map_augment
    ref.model.map_augment = None
    with torch.no_grad():
        for p in ref.parameters():  # the reference zero-initialises its output layers; make every part count
            p.add_(torch.randn_like(p) * 0.02)
    ours = config1_unet(1000)
    missing, unexpected = ours.load_state_dict(ref.state_dict(), strict=False)
    # the reference stores its fixed [1, 1] resampling filter as a buffer; here it is a constant
    assert not missing and all(k.endswith("resample_filter") for k in unexpected), (missing, unexpected)
    ref.eval(), ours.eval()
    g = torch.Generator().manual_seed(2)
    x = torch.randn(2, 3, 64, 64, generator=g)
    sigma = torch.tensor([0.3, 11.0])
    labels = torch.eye(1000)[torch.tensor([5, 999])]
    with torch.no_grad():
        torch.testing.assert_close(ours(x, sigma, labels), ref(x, sigma, labels), rtol=2e-4, atol=2e-4)
        rb = ref(x, sigma, labels, return_bottleneck=True)
        ob = ours(x, sigma, labels, return_bottleneck=True)
    torch.testing.assert_close(ob, rb, rtol=2e-4, atol=2e-4)
