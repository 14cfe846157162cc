"""Fused data-parallel optimiser kernels (csrc/collectives.cu) on B200.

* one GPU: the dp_adamw kernel (world 1) against the fp32 PyTorch AdamW of the same step,
  with clipping by the global norm and the EMA;
* one GPU: the bounded barrier gives up on a flag that nothing sets, reports status 5 and
  the optimiser kernel that follows leaves the weights untouched;
* two GPUs (skipped with fewer): ShardedAdamW over symmetric memory, P2P and NVLS paths,
  against a replicated AdamW on the rank-averaged gradients.
"""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _adamw_ref(w, g, m, v, step, lr, b1, b2, eps, wd, scale=1.0, ema=None, ema_beta=0.0):
    g = g.float() * scale
    w = w * (1 - lr * wd)
    m = b1 * m + (1 - b1) * g
    v = b2 * v + (1 - b2) * g * g
    bc1, bc2 = 1 - b1 ** step, 1 - b2 ** step
    w = w - lr / bc1 * m / ((v / bc2).sqrt() + eps)
    if ema is not None:
        ema = ema_beta * ema + (1 - ema_beta) * w
    return w, m, v, ema


@pytest.mark.parametrize("clip", [None, 0.25])
def test_dp_adamw_single_gpu(clip):
    from dmad_b200.ops import ext, check_device_status
    from dmad_b200.parallel.symm import PeerSync

    torch.manual_seed(0)
    n = 1 << 20
    dev = torch.device("cuda", 0)
    w0 = torch.randn(n, device=dev)
    p = w0.to(torch.bfloat16)
    g = torch.randn(n, device=dev).to(torch.bfloat16)
    master, m, v = w0.clone(), torch.randn(n, device=dev).abs() * 0.1, torch.rand(n, device=dev) * 0.01
    ema = w0.clone()
    m0, v0 = m.clone(), v.clone()
    slots = None
    scale = 1.0
    if clip is not None:
        acc = torch.zeros(1, device=dev)
        ext().dp_sumsq([g.data_ptr()], [p.data_ptr()], 0, 0, 2, 0, n, acc, False)
        ref_ss = float((g.float() ** 2).sum())
        assert abs(float(acc) - ref_ss) / ref_ss < 1e-4
        sync = PeerSync(dev)
        sync(acc)
        slots = sync.slots
        scale = min(1.0, clip / (ref_ss ** 0.5 + 1e-6))
    ext().dp_adamw([g.data_ptr()], [p.data_ptr()], 0, 0, 2, master, m, v, ema, 0, n, 1e-3, 0.9, 0.99, 1e-8,
                   0.01, 3, 0.95, slots, float(clip or 0.0), False)
    torch.cuda.synchronize()
    check_device_status()
    rw, rm, rv, re = _adamw_ref(w0, g, m0, v0, 3, 1e-3, 0.9, 0.99, 1e-8, 0.01, scale, w0.clone(), 0.95)
    torch.testing.assert_close(master, rw, rtol=1e-5, atol=1e-6)
    torch.testing.assert_close(m, rm, rtol=1e-5, atol=1e-7)
    torch.testing.assert_close(v, rv, rtol=1e-5, atol=1e-9)
    torch.testing.assert_close(ema, re, rtol=1e-5, atol=1e-6)
    # the bf16 weights are exactly the kernel's fp32 master rounded
    torch.testing.assert_close(p.float(), master.to(torch.bfloat16).float(), rtol=0, atol=0)


def test_barrier_timeout_reports_and_blocks_update():
    """A peer flag that nothing sets: the wait gives up after its limit, the status word says
    so, and the optimiser kernel behind it skips its update."""
    from dmad_b200.ops import ext, device_status

    dev = torch.device("cuda", 0)
    device_status(0, reset=True)
    mine = torch.zeros(8, dtype=torch.int32, device=dev)
    fake_peer = torch.zeros(8, dtype=torch.int32, device=dev)  # stands for rank 1's buffer
    ptrs = torch.tensor([mine.data_ptr(), fake_peer.data_ptr()], dtype=torch.int64, device=dev)
    ext().symm_barrier(ptrs, 0, 1, None, 0.5)  # rank 1 never writes mine[1]
    n = 4096
    p = torch.ones(n, dtype=torch.bfloat16, device=dev)
    g = torch.ones(n, dtype=torch.bfloat16, device=dev)
    master, m, v = torch.ones(n, device=dev), torch.zeros(n, device=dev), torch.zeros(n, device=dev)
    ext().dp_adamw([g.data_ptr()], [p.data_ptr()], 0, 0, 2, master, m, v, None, 0, n, 1e-2, 0.9, 0.99, 1e-8,
                   0.0, 1, 0.0, None, 0.0, False)
    torch.cuda.synchronize()
    assert int(fake_peer[0]) == 1  # our own flag reached the peer
    assert device_status(0, reset=True) == 5
    assert float(master.min()) == 1.0 and float(master.max()) == 1.0
    assert float(m.abs().max()) == 0.0


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _make(seed):
    g = torch.Generator().manual_seed(seed)
    return [torch.randn(s, generator=g) for s in [(257, 33), (4099,), (64, 64), (1000, 3)]]


def _grad(rank, step, shapes):
    g = torch.Generator().manual_seed(10 * step + rank)
    return [torch.randn(s, generator=g) for s in shapes]


def _worker(rank, world, port, multicast, clip, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank), NCCL_NVLS_ENABLE="0")
    try:
        import torch.distributed as dist
        from dmad_b200.ops import check_device_status
        from dmad_b200.parallel.dist import init_distributed
        from dmad_b200.parallel.zero import ShardedAdamW

        _, _, dev = init_distributed(timeout_s=60)
        params = [torch.nn.Parameter(t.to(dev, torch.bfloat16)) for t in _make(0)]
        opt = ShardedAdamW(params, lr=1e-2, betas=(0.9, 0.99), weight_decay=0.01, ema=True,
                           use_multicast=multicast, sync_timeout_s=10.0)
        used_mc = opt.multicast
        for s in range(3):
            opt.zero_grad()
            for p, g in zip(params, _grad(rank, s, [p.shape for p in params])):
                p.grad.add_(g.to(dev, torch.bfloat16))
            opt.step(ema_beta=0.9, max_grad_norm=clip)
        torch.cuda.synchronize()
        check_device_status()
        # numpy arrays: tensors sent through the queue would need the worker alive to be received
        out = [p.detach().float().cpu().numpy() for p in params]
        ema = [e.cpu().numpy() for e in opt.full_ema()]
        master = [m_.cpu().numpy() for m_ in opt.full_master()]
        del opt
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, out, ema, master, used_mc, None))
    except Exception as e:  # pragma: no cover
        q.put((rank, None, None, None, None, repr(e)))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("multicast,clip", [(False, None), (False, 1.0), (True, None)])
def test_sharded_adamw_two_gpus(multicast, clip):
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, multicast, clip, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    # replicated reference: bf16 weights / grads as the GPUs hold them, fp32 math
    shapes = [t.shape for t in _make(0)]
    w = [t.to(torch.bfloat16).float() for t in _make(0)]
    m = [torch.zeros_like(t) for t in w]
    v = [torch.zeros_like(t) for t in w]
    ema = [t.clone() for t in w]
    for s in range(3):
        grads = [sum(gs) / world for gs in zip(*[[g.to(torch.bfloat16).float() for g in _grad(r, s, shapes)]
                                                  for r in range(world)])]
        scale = 1.0
        if clip is not None:
            n = float(torch.sqrt(sum((g * g).sum() for g in grads)))
            scale = min(1.0, clip / (n + 1e-6))
        for i in range(len(w)):
            w[i], m[i], v[i], ema[i] = _adamw_ref(w[i], grads[i], m[i], v[i], s + 1, 1e-2, 0.9, 0.99, 1e-8, 0.01,
                                                  scale, ema[i], 0.9)
    for rank, out, e_out, master, used_mc, err in res:
        assert err is None, err
        out, e_out, master = ([torch.from_numpy(a) for a in xs] for xs in (out, e_out, master))
        tol = 2e-2 if used_mc else 1e-4  # the switch returns bf16 sums
        for a, b in zip(master, w):
            torch.testing.assert_close(a, b, rtol=tol, atol=tol)
        for a, b in zip(out, master):
            torch.testing.assert_close(a, b.to(torch.bfloat16).float(), rtol=0, atol=0)
        for a, b in zip(e_out, ema):
            torch.testing.assert_close(a, b, rtol=tol, atol=tol)
