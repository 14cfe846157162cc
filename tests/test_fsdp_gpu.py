"""Sharded frozen block weights on 2 GPUs (skipped with fewer): peer-pull gathers one block ahead on a
side stream reproduce the unsharded LoRA-student forward and LoRA gradients (the gathered weights are
bit-identical; the GEMM library may pick other kernels for the differently aligned views, so the
results are compared within bf16 tolerance)."""
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
    m = WanModel(WanConfig(dim=256, ffn_dim=512, num_heads=2, num_layers=4, text_dim=64, freq_dim=64))
    torch.nn.init.normal_(m.head.head.weight, std=0.05)
    m.enable_lora(16)
    for b in m.blocks:
        for lin in b.linears():
            torch.nn.init.normal_(lin.lora_B, std=0.02)
    m = m.to(dev, torch.bfloat16)
    m.checkpoint_blocks = 4
    return m.train()


def _run(m, dev):
    g = torch.Generator().manual_seed(5)
    x = torch.randn(1, 16, 4, 16, 16, generator=g).to(dev)
    t, ctx = torch.rand(1, 1, generator=g).to(dev), torch.randn(1, 24, 64, generator=g).to(dev)
    out = m(x, t, ctx)
    out.float().square().mean().backward()
    grads = torch.cat([p.grad.float().reshape(-1) for p in m.parameters() if p.grad is not None])
    return out.detach().float(), grads


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank), NCCL_NVLS_ENABLE="0")
    try:
        import torch.distributed as dist
        from dmad_b200.ops import check_device_status
        from dmad_b200.parallel.dist import init_distributed
        from dmad_b200.parallel.fsdp import ShardedFrozenBlocks

        _, _, dev = init_distributed(timeout_s=60)
        m = _model(dev)
        ShardedFrozenBlocks(m.blocks)
        out, grads = _run(m, dev)
        torch.cuda.synchronize()
        check_device_status()
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, out.cpu().numpy(), grads.cpu().numpy(), None))
    except Exception:  # pragma: no cover
        import traceback
        q.put((rank, None, None, traceback.format_exc()))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_sharded_frozen_blocks_two_gpus():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    dev = torch.device("cuda", 0)
    out, grads = _run(_model(dev), dev)
    for rank, o, g, err in res:
        assert err is None, err
        o, g = torch.from_numpy(o).to(dev), torch.from_numpy(g).to(dev)
        assert (o - out).abs().max().item() < 2e-2 * max(1.0, out.abs().max().item())
        assert ((g - grads).norm() / grads.norm()).item() < 2e-2


def _worker_trainable(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank), NCCL_NVLS_ENABLE="0")
    try:
        import torch.distributed as dist
        from dmad_b200.models.wan import WanConfig, WanModel
        from dmad_b200.ops import check_device_status
        from dmad_b200.parallel.dist import init_distributed
        from dmad_b200.parallel.fsdp import ShardedTrainableBlocks

        _, _, dev = init_distributed(timeout_s=60)
        torch.manual_seed(0)
        m = WanModel(WanConfig(dim=256, ffn_dim=512, num_heads=2, num_layers=4, text_dim=64, freq_dim=64))
        torch.nn.init.normal_(m.head.head.weight, std=0.05)
        m = m.to(dev, torch.bfloat16).train()
        m.checkpoint_blocks = 4
        full0 = [p.detach().clone() for b in m.blocks for p in b.parameters()]
        sh = ShardedTrainableBlocks(m.blocks, lr=1e-3, betas=(0.9, 0.99), weight_decay=0.01)
        # (1) the peer-pull gather equals NCCL's all-gather of the shards, bit for bit
        gathered = torch.cat([t.reshape(-1) for t in sh.full_params()])
        ok_gather = torch.equal(gathered, torch.cat([t.reshape(-1) for t in full0]))
        ps, offs, n, ln, base = sh.layout[1]
        ref = torch.empty(ln * world, dtype=torch.bfloat16, device=dev)
        dist.all_gather_into_tensor(ref, sh.arena.tensor[base:base + ln].contiguous())
        sh._gather(1, 0)
        torch.cuda.synchronize()
        ok_gather = ok_gather and torch.equal(sh.slots[0][:ln * world], ref)
        # (2) the reduce-scatter kernel equals NCCL's reduce-scatter (fp32 sum of the bf16 gradients)
        g = torch.Generator(device=dev).manual_seed(50 + rank)
        grad = torch.randn(ln * world, generator=g, device=dev).to(torch.bfloat16)
        sh.gslots.tensor[:ln * world].copy_(grad)
        sh.grad_acc.zero_()
        sh._reduce_scatter(1, 0)
        mine = sh.grad_acc[base:base + ln].clone()
        nccl = torch.empty(ln, dtype=torch.float32, device=dev)
        dist.reduce_scatter_tensor(nccl, grad.float())
        ok_rs = torch.equal(mine, nccl)
        # (3) a training step end to end: each rank its own sample
        sh.zero_grad()
        gs = torch.Generator().manual_seed(7 + rank)
        x = torch.randn(1, 16, 4, 16, 16, generator=gs).to(dev)
        t, ctx = torch.rand(1, 1, generator=gs).to(dev), torch.randn(1, 24, 64, generator=gs).to(dev)
        m(x, t, ctx).float().square().mean().backward()
        sh.step()
        after = [t_.float().cpu() for t_ in sh.full_params()]
        torch.cuda.synchronize()
        check_device_status()
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, ok_gather, ok_rs, [a.numpy() for a in after], None))
    except Exception:  # pragma: no cover
        import traceback
        q.put((rank, None, None, None, traceback.format_exc()))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_sharded_trainable_blocks_two_gpus():
    """Trainable-weight sharding: the peer-memory gather and reduce-scatter kernels equal NCCL's
    all-gather / reduce-scatter bit for bit, and one sharded step matches replicated data-parallel
    training (the mean gradient of both ranks' samples, AdamW on full tensors) within bf16 tolerance."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker_trainable, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    for rank, ok_gather, ok_rs, after, err in res:
        assert err is None, err
        assert ok_gather and ok_rs, (rank, ok_gather, ok_rs)
    # replicated reference on one GPU
    from dmad_b200.models.wan import WanConfig, WanModel
    from dmad_b200.ops.optim import FusedAdamW

    dev = torch.device("cuda", 0)
    torch.manual_seed(0)
    m = WanModel(WanConfig(dim=256, ffn_dim=512, num_heads=2, num_layers=4, text_dim=64, freq_dim=64))
    torch.nn.init.normal_(m.head.head.weight, std=0.05)
    m = m.to(dev, torch.bfloat16).train()
    m.checkpoint_blocks = 4
    params = [p for b in m.blocks for p in b.parameters()]
    acc = [torch.zeros_like(p, dtype=torch.float32) for p in params]
    for r in range(2):
        gs = torch.Generator().manual_seed(7 + r)
        x = torch.randn(1, 16, 4, 16, 16, generator=gs).to(dev)
        t, ctx_ = torch.rand(1, 1, generator=gs).to(dev), torch.randn(1, 24, 64, generator=gs).to(dev)
        for p in m.parameters():
            p.grad = None
        m(x, t, ctx_).float().square().mean().backward()
        for a, p in zip(acc, params):
            a.add_(p.grad.float())
    opt = FusedAdamW(params, lr=1e-3, betas=(0.9, 0.99), weight_decay=0.01)
    for a, p in zip(acc, params):
        p.grad = (a / 2).to(torch.bfloat16)
    opt.step()
    for rank, ok_gather, ok_rs, after, err in res:
        for a, p in zip(after, params):
            ref = p.detach().float().cpu()
            assert (torch.from_numpy(a) - ref).abs().max().item() <= 2e-2 * max(1.0, ref.abs().max().item())
