"""Ring attention (impl="ring") on 2 gloo CPU ranks: the per-block LSE merge reproduces the
unsharded Wan forward and its gradients, and the per-block (O, T~/l, mu) merge its JVP."""
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


def _model():
    from dmad_b200.models.wan import WanConfig, WanModel

    torch.manual_seed(0)
    m = WanModel(WanConfig(dim=256, ffn_dim=512, num_heads=2, num_layers=2, text_dim=32, freq_dim=64))
    torch.nn.init.normal_(m.head.head.weight, std=0.05)
    return m


def _inputs():
    g = torch.Generator().manual_seed(7)
    return torch.randn(2, 16, 2, 4, 8, generator=g), torch.rand(2, 1, generator=g), torch.randn(2, 5, 32, generator=g)


def _jvp_inputs():
    g = torch.Generator().manual_seed(9)
    x, t, ctx = _inputs()
    return x, torch.randn(x.shape, generator=g), t, torch.rand(2, 1, generator=g), ctx


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    try:
        import torch.distributed as dist
        from dmad_b200.parallel.cp import ContextParallel
        from dmad_b200.parallel.dist import init_distributed

        init_distributed(backend="gloo", timeout_s=120)
        m = _model()
        m.enable_context_parallel(ContextParallel(impl="ring"))
        from dmad_b200.models.wan_jvp import wan_forward_jvp

        out = m(*_inputs())
        out.square().sum().backward()
        grads = torch.cat([p.grad.reshape(-1) for p in m.parameters()])
        dist.all_reduce(grads)  # parameter gradients summed over the CP group
        with torch.no_grad():
            jo, jt = wan_forward_jvp(m, *_jvp_inputs())
        q.put((rank, (out.detach().numpy(), jo.numpy(), jt.numpy(), grads.numpy()), None))
        dist.destroy_process_group()
    except Exception:  # pragma: no cover
        import traceback
        q.put((rank, None, traceback.format_exc()))


def test_ring_matches_unsharded():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    from dmad_b200.models.wan_jvp import wan_forward_jvp

    m = _model()
    out = m(*_inputs())
    out.square().sum().backward()
    grads = torch.cat([p.grad.reshape(-1) for p in m.parameters()])
    out = out.detach()
    with torch.no_grad():
        jo, jt = wan_forward_jvp(m, *_jvp_inputs())
    for rank, o, err in res:
        assert err is None, err
        torch.testing.assert_close(torch.from_numpy(o[0]), out, rtol=1e-4, atol=1e-5)
        torch.testing.assert_close(torch.from_numpy(o[1]), jo, rtol=1e-4, atol=1e-5)
        torch.testing.assert_close(torch.from_numpy(o[2]), jt, rtol=1e-3, atol=1e-5)
        torch.testing.assert_close(torch.from_numpy(o[3]), grads, rtol=1e-3, atol=1e-5)
