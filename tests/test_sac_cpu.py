"""Activation checkpointing policies (block_wise, mm_only) of the Wan blocks: same gradients as no
checkpointing; mm_only runs no matrix product again in the backward, block_wise runs them all again
(parity: train/wan/rcm/utils/selective_activation_checkpoint.py:26-74)."""
import pytest
import torch
from torch.utils._python_dispatch import TorchDispatchMode


class _CountMM(TorchDispatchMode):
    def __init__(self):
        super().__init__()
        self.n = 0

    def __torch_dispatch__(self, func, types, args=(), kwargs=None):
        if func in (torch.ops.aten.mm.default, torch.ops.aten.addmm.default, torch.ops.aten.bmm.default):
            self.n += 1
        return func(*args, **(kwargs or {}))


def _model():
    from dmad_b200.models.wan import WanConfig, WanModel

    torch.manual_seed(0)
    m = WanModel(WanConfig(dim=128, ffn_dim=256, num_heads=2, num_layers=2, text_dim=32, freq_dim=64))
    torch.nn.init.normal_(m.head.head.weight, std=0.05)
    return m.train()


def _inputs():
    g = torch.Generator().manual_seed(3)
    return torch.randn(1, 16, 2, 4, 8, generator=g), torch.rand(1, 1, generator=g), torch.randn(1, 6, 32, generator=g)


def _grads(policy):
    m = _model()
    if policy is not None:
        m.checkpoint_blocks = len(m.blocks)
        m.checkpoint_policy = policy
    out = m(*_inputs())
    loss = out.square().mean()
    with _CountMM() as c:
        loss.backward()
    return torch.cat([p.grad.reshape(-1) for p in m.parameters() if p.grad is not None]), c.n


@pytest.mark.parametrize("policy", ["block_wise", "mm_only"])
def test_checkpoint_policies_match(policy):
    g0, n0 = _grads(None)
    g, n = _grads(policy)
    torch.testing.assert_close(g, g0, rtol=1e-5, atol=1e-6)
    if policy == "mm_only":
        assert n == n0, (n, n0)  # the backward's own products only: none recomputed
    else:
        assert n > n0, (n, n0)


def test_unknown_policy():
    from dmad_b200.models.sac import checkpoint_block

    with pytest.raises(ValueError):
        checkpoint_block(lambda x: x * 2, torch.ones(2, requires_grad=True), policy="nope")
