"""The fused spectral-norm kernels of SegLinear against the PyTorch restatement of the same math
(fp32 power iteration on the weight, sigma differentiable in W with u and v held constant)."""
import copy

import pytest
import torch

pytestmark = pytest.mark.gpu


def _layer(zero_seg):
    from dmad_b200.models.layers import SegLinear

    torch.manual_seed(0)
    lin = SegLinear(512, [("q", 256), ("k", 128), ("v", 384)], bias=True, flat_name="qkv")
    with torch.no_grad():
        if zero_seg:
            lin.weight[256:384].zero_()  # a zero-initialised segment: no norm on it
    lin.enable_spectral_norm(3)
    return lin.to("cuda", torch.bfloat16)


def _reference_weight(lin):
    return (lin.weight.float() * lin._sn_row_scale()[:, None]).to(lin.weight.dtype)


@pytest.mark.parametrize("train", [True, False])
@pytest.mark.parametrize("zero_seg", [False, True])
def test_fused_spectral_norm_matches_pytorch(train, zero_seg):
    fused = _layer(zero_seg)
    ref = copy.deepcopy(fused)
    fused.train(train)
    ref.train(train)
    assert fused._sn_segments_on() == [True, not zero_seg, True]
    for it in range(3):  # the power-iteration state carries over between forwards
        wf = fused.effective_weight()
        wr = _reference_weight(ref)
        torch.cuda.synchronize()
        assert (wf.float() - wr.float()).abs().max().item() <= 2e-2 * wr.float().abs().max().item()
        torch.testing.assert_close(fused.sn_u.float(), ref.sn_u.float(), rtol=2e-3, atol=2e-4)
        torch.testing.assert_close(fused.sn_v.float(), ref.sn_v.float(), rtol=2e-3, atol=2e-4)
        # gradient through sigma and the scale
        g = torch.randn(wf.shape, device="cuda", generator=torch.Generator("cuda").manual_seed(it)).to(wf.dtype)
        (dwf,) = torch.autograd.grad((wf.float() * g.float()).sum(), fused.weight)
        (dwr,) = torch.autograd.grad((wr.float() * g.float()).sum(), ref.weight)
        rel = (dwf.float() - dwr.float()).norm() / dwr.float().norm()
        assert rel < 2e-2, (it, rel.item())


def test_fused_spectral_norm_in_forward_and_state_dict():
    """The layer's forward uses the fused weight; a state-dict round trip carries the norm state and the
    segment mask (a segment that was off in the target is on after loading)."""
    lin = _layer(False).train()
    x = torch.randn(64, 512, device="cuda", dtype=torch.bfloat16)
    y = lin(x)
    y.float().square().mean().backward()
    assert lin.weight.grad is not None and torch.isfinite(lin.weight.grad.float()).all()
    other = _layer(True)
    assert other._sn_segments_on() == [True, False, True]
    other.load_state_dict(lin.state_dict())
    assert other._sn_segments_on() == [True, True, True]
    other.eval()
    lin.eval()
    torch.testing.assert_close(other.effective_weight().float(), lin.effective_weight().float())
