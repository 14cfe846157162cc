"""Sharded frozen block weights on 2 gloo CPU ranks: a LoRA-student Wan model whose frozen block
weights are sharded (gathered one block ahead, activation checkpointing) gives the same output and
LoRA gradients as the unsharded model."""
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
    m = WanModel(WanConfig(dim=128, ffn_dim=256, num_heads=1, num_layers=3, text_dim=32, freq_dim=64))
    torch.nn.init.normal_(m.head.head.weight, std=0.05)
    m.enable_lora(8)
    for b in m.blocks:
        for lin in b.linears():
            torch.nn.init.normal_(lin.lora_B, std=0.02)
    m = m.to(torch.bfloat16)
    m.checkpoint_blocks = 3
    m.train()
    return m


def _run(m):
    g = torch.Generator().manual_seed(5)
    x, t, ctx = torch.randn(1, 16, 2, 4, 4, generator=g), torch.rand(1, 1, generator=g), torch.randn(1, 8, 32, generator=g)
    out = m(x.bfloat16(), t, ctx.bfloat16())
    out.float().square().mean().backward()
    grads = torch.cat([p.grad.float().reshape(-1) for n, p in m.named_parameters() if p.grad is not None])
    return out.detach().float(), grads


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    try:
        import torch.distributed as dist
        from dmad_b200.parallel.dist import init_distributed
        from dmad_b200.parallel.fsdp import ShardedFrozenBlocks

        init_distributed(backend="gloo", timeout_s=120)
        m = _model()
        sh = ShardedFrozenBlocks(m.blocks)
        assert all(p.numel() == 0 for b in m.blocks for p in b.parameters() if not p.requires_grad
                   and p.dtype == torch.bfloat16)
        out, grads = _run(m)
        q.put((rank, out.numpy(), grads.numpy(), sh.arena.tensor.numel(), None))
        dist.destroy_process_group()
    except Exception:  # pragma: no cover
        import traceback
        q.put((rank, None, None, None, traceback.format_exc()))


def test_sharded_frozen_blocks_match():
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
    m = _model()
    out, grads = _run(m)
    full = sum(p.numel() for b in m.blocks for p in b.parameters() if not p.requires_grad and p.dtype == torch.bfloat16)
    for rank, o, g, shard_elems, err in res:
        assert err is None, err
        assert shard_elems < 0.6 * full
        torch.testing.assert_close(torch.from_numpy(o), out, rtol=0, atol=0)
        torch.testing.assert_close(torch.from_numpy(g), grads, rtol=0, atol=0)
