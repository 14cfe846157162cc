"""Sharded data-parallel AdamW on gloo CPU ranks.

The sharded optimiser (flat buffers, per-rank fp32 shards, host path of the fused
reduce-scatter / update / all-gather) must produce the same weights as a replicated AdamW
fed the rank-averaged gradients, with and without clipping by the global norm, and its EMA
gathered from the shards must match a replicated EMA."""
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


def _make_params(seed):
    g = torch.Generator().manual_seed(seed)
    shapes = [(7, 5), (13,), (3, 4, 2), (33,)]
    return [torch.nn.Parameter(torch.randn(s, generator=g)) for s in shapes]


def _grads(rank, step, params):
    g = torch.Generator().manual_seed(1000 * step + rank)
    return [torch.randn(p.shape, generator=g) * (3.0 if step == 1 else 1.0) for p in params]


def _reference(world, steps, clip, lr=1e-2, betas=(0.9, 0.99), wd=0.05, ema_beta=0.9):
    from dmad_b200.ops.optim import FusedAdamW

    params = _make_params(0)
    ema = [p.detach().clone() for p in params]
    opt = FusedAdamW(params, lr=lr, betas=betas, weight_decay=wd, ema=ema)
    for s in range(steps):
        per_rank = [_grads(r, s, params) for r in range(world)]
        for i, p in enumerate(params):
            p.grad = sum(pr[i] for pr in per_rank) / world
        opt.step(ema_beta=ema_beta, max_grad_norm=clip)
    return [p.detach().clone() for p in params], ema


def _worker(rank, world, port, steps, clip, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    try:
        from dmad_b200.parallel.dist import init_distributed
        from dmad_b200.parallel.zero import ShardedAdamW

        init_distributed(backend="gloo", timeout_s=120)
        params = _make_params(0)
        opt = ShardedAdamW(params, lr=1e-2, betas=(0.9, 0.99), weight_decay=0.05, ema=True)
        for s in range(steps):
            opt.zero_grad()
            for p, g in zip(params, _grads(rank, s, params)):
                p.grad.add_(g)  # accumulate into the flat-buffer view, as autograd does
            opt.step(ema_beta=0.9, max_grad_norm=clip)
        # numpy arrays: tensors sent through the queue would need the worker alive to be received
        ema = [e.numpy() for e in opt.full_ema()]
        q.put((rank, [p.detach().numpy().copy() for p in params], ema, None))
        dist.destroy_process_group()
    except Exception as e:  # pragma: no cover
        q.put((rank, None, None, repr(e)))


@pytest.mark.parametrize("clip", [None, 0.5])
def test_sharded_adamw_matches_replicated(clip):
    world, steps = 2, 3
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, steps, clip, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    ref_w, ref_ema = _reference(world, steps, clip)
    for rank, w, ema, err in res:
        assert err is None, err
        for a, b in zip(w, ref_w):
            torch.testing.assert_close(torch.from_numpy(a), b, rtol=1e-5, atol=1e-6)
        for a, b in zip(ema, ref_ema):
            torch.testing.assert_close(torch.from_numpy(a), b, rtol=1e-5, atol=1e-6)


def test_flat_views_single_process():
    from dmad_b200.parallel.zero import ShardedAdamW

    params = _make_params(3)
    before = [p.detach().clone() for p in params]
    opt = ShardedAdamW(params, lr=1e-2)
    g = opt.groups[0]
    for p, b, o in zip(params, before, g.offsets):
        assert torch.equal(p.detach(), b)
        assert p.data.data_ptr() == g.pbuf.tensor[o:].data_ptr()
        assert o % 8 == 0
    # autograd accumulates into the flat gradient buffer in place
    loss = sum((p * p).sum() for p in params)
    loss.backward()
    for p, o in zip(params, g.offsets):
        assert p.grad.data_ptr() == g.gbuf.tensor[o:].data_ptr()
        torch.testing.assert_close(p.grad, 2 * p.detach())
    opt.step()
    opt.zero_grad()
    assert float(g.gbuf.tensor.abs().sum()) == 0.0
    assert all(p.grad is not None for p in params)


def _np_tree(x):
    if torch.is_tensor(x):
        return ("__t__", x.detach().cpu().numpy())
    if isinstance(x, dict):
        return {k: _np_tree(v) for k, v in x.items()}
    if isinstance(x, (list, tuple)):
        return [_np_tree(v) for v in x]
    return x


def _torch_tree(x):
    if isinstance(x, tuple) and len(x) == 2 and x[0] == "__t__":
        return torch.from_numpy(x[1])
    if isinstance(x, list) and len(x) == 2 and x[0] == "__t__":
        return torch.from_numpy(x[1])
    if isinstance(x, dict):
        return {k: _torch_tree(v) for k, v in x.items()}
    if isinstance(x, list):
        return [_torch_tree(v) for v in x]
    return x


def _elastic_worker(rank, world, port, mode, states, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    try:
        from dmad_b200.parallel.dist import init_distributed
        from dmad_b200.parallel.zero import ShardedAdamW

        init_distributed(backend="gloo", timeout_s=120)
        params = _make_params(0 if mode == "train" else 5)
        opt = ShardedAdamW(params, lr=1e-2, betas=(0.9, 0.99), weight_decay=0.05, ema=True)
        if mode == "train":
            for s in range(3):
                opt.zero_grad()
                for p, g in zip(params, _grads(rank, s, params)):
                    p.grad.add_(g)
                opt.step(ema_beta=0.9)
        else:
            opt.load_resharded([_torch_tree(st) for st in states])
        out = (_np_tree(opt.state_dict()), [m.numpy() for m in opt.full_master()], [e.numpy() for e in opt.full_ema()],
               [p.detach().numpy() for p in params], opt.step_count)
        q.put((rank, out, None))
        dist.destroy_process_group()
    except Exception:  # pragma: no cover
        import traceback
        q.put((rank, None, traceback.format_exc()))


def _spawn(world, mode, states=None):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_elastic_worker, args=(r, world, port, mode, states, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted([q.get(timeout=300) for _ in procs], key=lambda r: r[0])
    for p in procs:
        p.join(timeout=60)
    for _, _, err in res:
        assert err is None, err
    return [r[1] for r in res]


def test_elastic_resume_reshards_optimizer_state():
    """Shard states of a 2-rank run reloaded on 3 ranks and on 1 process: the same full fp32 master and
    EMA, the same bf16/fp32 weights and step count."""
    from dmad_b200.parallel.zero import ShardedAdamW

    old = _spawn(2, "train")
    states = [o[0] for o in old]
    full_m, full_e, weights, step = old[0][1], old[0][2], old[0][3], old[0][4]
    new = _spawn(3, "load", states)
    for _, m, e, w, st in new:
        assert st == step
        for a, b in zip(m + e + w, full_m + full_e + weights):
            np_a, np_b = torch.from_numpy(a), torch.from_numpy(b)
            torch.testing.assert_close(np_a, np_b)
    params = _make_params(9)
    opt = ShardedAdamW(params, lr=1e-2, ema=True)
    opt.load_resharded([_torch_tree(st) for st in states])
    for a, b in zip(opt.full_master() + [p.detach() for p in params], full_m + weights):
        torch.testing.assert_close(a, torch.from_numpy(b))
