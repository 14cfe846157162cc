"""Ulysses context parallelism on 2 gloo CPU ranks: the sequence-sharded Wan forward (all-to-all
around self-attention, all-gather of the head output) and its parameter gradients summed over the
CP group must equal the unsharded model's, for uniform and per-frame timesteps, and the CP-pooled
critic logits must equal the unsharded pooling."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _model():
    from dmad_b200.models.wan import WanConfig, WanModel

    torch.manual_seed(0)
    m = WanModel(WanConfig(dim=256, ffn_dim=512, num_heads=2, num_layers=2, text_dim=32, freq_dim=64))
    # non-zero head so the output depends on every block
    torch.nn.init.normal_(m.head.head.weight, std=0.05)
    return m


def _inputs(per_frame):
    g = torch.Generator().manual_seed(7)
    x = torch.randn(2, 16, 2, 4, 8, generator=g)  # L = 2 * 2 * 4 = 16 tokens
    t = torch.rand(2, 2, generator=g) if per_frame else torch.rand(2, 1, generator=g)
    ctx = torch.randn(2, 5, 32, generator=g)
    return x, t, ctx


def _worker(rank, world, port, per_frame, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    try:
        from dmad_b200.parallel.cp import ContextParallel
        from dmad_b200.parallel.dist import init_distributed

        init_distributed(backend="gloo", timeout_s=120)
        m = _model()
        m.enable_context_parallel(ContextParallel(impl="nccl"))
        x, t, ctx = _inputs(per_frame)
        out, feats = m(x, t, ctx, feature_hook_block=-1)
        (out.square().sum() + feats.sum()).backward()
        grads = torch.cat([p.grad.reshape(-1) for p in m.parameters()])
        dist.all_reduce(grads)  # parameter gradients summed over the CP group
        pooled = m.cp.all_reduce_sum(feats.mean(dim=1)) / m.cp.world
        from dmad_b200.models.wan_jvp import wan_forward_jvp
        g = torch.Generator().manual_seed(11)
        tx = torch.randn(x.shape, generator=g)
        tt = torch.rand(t.shape, generator=g)
        jo, jt = wan_forward_jvp(m, x, tx, t, tt, ctx)
        q.put((rank, out.detach().numpy(), grads.numpy(), pooled.detach().numpy(),
               (jo.numpy(), jt.numpy()), None))
        dist.destroy_process_group()
    except Exception as e:  # pragma: no cover
        import traceback
        q.put((rank, None, None, None, None, traceback.format_exc()))


@pytest.mark.parametrize("per_frame", [False, True])
def test_cp_matches_unsharded(per_frame):
    world = 2
    ctx_mp = mp.get_context("spawn")
    q = ctx_mp.Queue()
    port = _free_port()
    procs = [ctx_mp.Process(target=_worker, args=(r, world, port, per_frame, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    m = _model()
    x, t, ctx = _inputs(per_frame)
    out, feats = m(x, t, ctx, feature_hook_block=-1)
    (out.square().sum() + feats.sum()).backward()
    ref_grads = torch.cat([p.grad.reshape(-1) for p in m.parameters()])
    from dmad_b200.models.wan_jvp import wan_forward_jvp
    gj = torch.Generator().manual_seed(11)
    tx = torch.randn(x.shape, generator=gj)
    tt = torch.rand(t.shape, generator=gj)
    rjo, rjt = wan_forward_jvp(m, x, tx, t, tt, ctx)
    for rank, o, g, pooled, jvp, err in res:
        assert err is None, err
        o, g, pooled = torch.from_numpy(o), torch.from_numpy(g), torch.from_numpy(pooled)
        torch.testing.assert_close(torch.from_numpy(jvp[0]), rjo, rtol=1e-4, atol=1e-5)
        torch.testing.assert_close(torch.from_numpy(jvp[1]), rjt, rtol=1e-3, atol=1e-5)
        torch.testing.assert_close(o, out.detach(), rtol=1e-4, atol=1e-5)
        torch.testing.assert_close(g, ref_grads, rtol=1e-3, atol=1e-5)
        torch.testing.assert_close(pooled, feats.detach().mean(dim=1), rtol=1e-4, atol=1e-5)
