"""Hybrid context parallelism (Ulysses inside groups of 2, ring across 2 groups) on 4 gloo CPU ranks:
the Wan forward, its parameter gradients, its JVP and the padded H3 forward equal the unsharded model's."""
import os
import socket

import torch
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _wan():
    from dmad_b200.models.wan import WanConfig, WanModel

    torch.manual_seed(0)
    m = WanModel(WanConfig(dim=256, ffn_dim=512, num_heads=2, num_layers=2, text_dim=32, freq_dim=64))
    torch.nn.init.normal_(m.head.head.weight, std=0.05)
    return m


def _wan_inputs():
    g = torch.Generator().manual_seed(7)
    x = torch.randn(1, 16, 2, 4, 8, generator=g)  # 16 tokens over 4 ranks
    t, ctx = torch.rand(1, 1, generator=g), torch.randn(1, 5, 32, generator=g)
    tx, tt = torch.randn(x.shape, generator=g), torch.rand(1, 1, generator=g)
    return x, t, ctx, tx, tt


def _wan_run(m):
    from dmad_b200.models.wan_jvp import wan_forward_jvp

    x, t, ctx, tx, tt = _wan_inputs()
    out = m(x, t, ctx)
    out.square().sum().backward()
    grads = torch.cat([p.grad.reshape(-1) for p in m.parameters()])
    jo, jt = wan_forward_jvp(m, x, tx, t, tt, ctx)
    return out.detach(), grads, jt


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    try:
        import torch.distributed as dist

        from dmad_b200.parallel.cp import HybridContextParallel
        from dmad_b200.parallel.dist import init_distributed
        from test_h3_cp_cpu import _setup as h3_setup

        init_distributed(backend="gloo", timeout_s=120)
        hcp = HybridContextParallel(ulysses_size=2)
        assert (hcp.u, hcp.r, hcp.ulysses.world, hcp.ring.world) == (2, 2, 2, 2)
        m = _wan()
        m.enable_context_parallel(hcp)
        out, grads, jt = _wan_run(m)
        dist.all_reduce(grads)
        h3, kw, L = h3_setup()
        h3.enable_context_parallel(hcp)
        with torch.no_grad():
            v, a = h3(**kw)
        q.put((rank, out.numpy(), grads.numpy(), jt.numpy(), v.numpy(), a.numpy(), None))
        dist.destroy_process_group()
    except Exception:  # pragma: no cover
        import traceback
        q.put((rank, None, None, None, None, None, traceback.format_exc()))


def test_hybrid_cp_matches_unsharded():
    import sys
    sys.path.insert(0, os.path.dirname(__file__))
    world = 4
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    from test_h3_cp_cpu import _setup as h3_setup

    out, grads, jt = _wan_run(_wan())
    h3, kw, _ = h3_setup()
    with torch.no_grad():
        v, a = h3(**kw)
    for rank, o, g, j, vv, aa, err in res:
        assert err is None, err
        torch.testing.assert_close(torch.from_numpy(o), out, rtol=1e-4, atol=1e-5)
        torch.testing.assert_close(torch.from_numpy(g), grads, rtol=1e-3, atol=1e-5)
        torch.testing.assert_close(torch.from_numpy(j), jt, rtol=1e-3, atol=1e-5)
        torch.testing.assert_close(torch.from_numpy(vv), v, rtol=1e-4, atol=1e-5)
        torch.testing.assert_close(torch.from_numpy(aa), a, rtol=1e-4, atol=1e-5)
