"""Data-parallel DMAD on 2 gloo CPU ranks: the replicas must stay bit-identical after steps,
the gap statistics are all-reduced, and a rank that raises is reported (host-side failure)."""
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


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    try:
        from dmad_b200.distill.wan_dmad import WanDMAD, WanDMADConfig
        from dmad_b200.models.wan import WanConfig
        from dmad_b200.parallel.dist import init_distributed

        init_distributed(backend="gloo", timeout_s=120)
        cfg = WanDMADConfig(net=WanConfig(dim=128, ffn_dim=256, num_heads=1, num_layers=2, text_dim=32),
                            lr=1e-3, critic_lr=1e-3)
        m = WanDMAD(cfg, device="cpu", dtype=torch.float32, seed=rank)  # different seeds: broadcast must fix
        g = torch.Generator().manual_seed(100 + rank)                    # per-rank data
        batch = {"latents": torch.randn(1, 16, 2, 4, 4, generator=g),
                 "real_latents": torch.randn(1, 16, 2, 4, 4, generator=g),
                 "context": torch.randn(1, 8, 32, generator=g)}
        for it in range(4):
            m.training_step(batch, it)
        vec = torch.cat([p.detach().reshape(-1) for p in m.net.parameters()] +
                        [p.detach().reshape(-1) for p in m.net_fake_score.parameters()] + [m.gap.gap_ema])
        gathered = [torch.zeros_like(vec) for _ in range(world)]
        dist.all_gather(gathered, vec)
        q.put((rank, all(torch.equal(gathered[0], v) for v in gathered), float(m.gap.gap_ready.sum())))
        dist.destroy_process_group()
    except Exception as e:  # pragma: no cover
        q.put((rank, repr(e), -1))


def test_dp_replicas_stay_identical():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=600) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    for rank, same, ready in res:
        assert same is True, (rank, same)
        assert ready > 0
