"""Context parallelism on 2 GPUs (skipped with fewer): the fused peer-memory all-to-all kernels
(q/k norm + RoPE + push, flash epilogue scatter, backward peer copies) against the NCCL
all-to-all path and against the unsharded model on one GPU -- forward output, block features and
parameter gradients (summed over the CP group)."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _model(dev):
    from dmad_b200.models.wan import WanConfig, WanModel

    torch.manual_seed(0)
    m = WanModel(WanConfig(dim=512, ffn_dim=1024, num_heads=4, num_layers=2, text_dim=64, freq_dim=64))
    torch.nn.init.normal_(m.head.head.weight, std=0.05)
    return m.to(dev, torch.bfloat16)


def _inputs(dev, per_frame):
    g = torch.Generator().manual_seed(7)
    x = torch.randn(1, 16, 4, 16, 32, generator=g)  # L = 4 * 8 * 16 = 512 tokens
    t = torch.rand(1, 4, generator=g) if per_frame else torch.rand(1, 1, generator=g)
    ctx = torch.randn(1, 24, 64, generator=g)
    return x.to(dev), t.to(dev), ctx.to(dev)


def _run(m, dev, per_frame):
    from dmad_b200.models.wan_jvp import wan_forward_jvp

    x, t, ctx = _inputs(dev, per_frame)
    out, feats = m(x, t, ctx, feature_hook_block=-1)
    (out.float().square().mean() + feats.float().mean()).backward()
    grads = torch.cat([p.grad.float().reshape(-1) for p in m.parameters()])
    g = torch.Generator().manual_seed(3)
    tx = torch.randn(x.shape, generator=g).to(dev)
    tt = torch.rand(t.shape, generator=g).to(dev)
    _, jt = wan_forward_jvp(m, x, tx, t * 1000, tt * 1000, ctx)
    return out.detach().float(), feats.detach().float(), torch.cat([grads, jt.float().reshape(-1)])


def _worker(rank, world, port, impl, per_frame, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank), NCCL_NVLS_ENABLE="0")
    try:
        import torch.distributed as dist
        from dmad_b200.ops import check_device_status
        from dmad_b200.parallel.cp import ContextParallel
        from dmad_b200.parallel.dist import init_distributed

        _, _, dev = init_distributed(timeout_s=60)
        m = _model(dev)
        if impl.startswith("hybrid"):  # hybrid-u2: one Ulysses group of 2; hybrid-u1: a ring of 2
            from dmad_b200.parallel.cp import HybridContextParallel
            m.enable_context_parallel(HybridContextParallel(ulysses_size=int(impl[-1]), timeout_s=10.0))
        else:
            m.enable_context_parallel(ContextParallel(impl=impl, timeout_s=10.0))
        out, feats, grads = _run(m, dev, per_frame)
        torch.cuda.synchronize()
        check_device_status()
        n = sum(p.numel() for p in m.parameters())
        gpart = grads[:n].clone()
        dist.all_reduce(gpart)  # parameter gradients summed over the CP group; the JVP tail is full
        grads = torch.cat([gpart, grads[n:]])
        fl = [torch.empty_like(feats) for _ in range(world)]
        dist.all_gather(fl, feats.contiguous())
        feats_full = torch.cat(fl, dim=1)
        m.enable_context_parallel(None)
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, out.cpu().numpy(), feats_full.cpu().numpy(), grads.cpu().numpy(), None))
    except Exception:  # pragma: no cover
        import traceback
        q.put((rank, None, None, None, traceback.format_exc()))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("impl,per_frame", [("fused", False), ("nccl", False), ("fused", True), ("ring", False),
                                            ("hybrid-u2", False), ("hybrid-u1", False)])
def test_cp_two_gpus_matches_unsharded(impl, per_frame):
    world = 2
    ctx_mp = mp.get_context("spawn")
    q = ctx_mp.Queue()
    port = _free_port()
    procs = [ctx_mp.Process(target=_worker, args=(r, world, port, impl, per_frame, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    dev = torch.device("cuda", 0)
    m = _model(dev)
    out, feats, grads = _run(m, dev, per_frame)
    for rank, o, f, g, err in res:
        assert err is None, err
        o, f, g = (torch.from_numpy(a).to(dev) for a in (o, f, g))
        assert (o - out).abs().max().item() < 3e-2 * max(1.0, out.abs().max().item())
        assert (f - feats).abs().max().item() < 3e-2 * max(1.0, feats.abs().max().item())
        rel = (g - grads).norm() / grads.norm()
        assert rel.item() < 2e-2, rel.item()
