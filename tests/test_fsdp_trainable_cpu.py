"""Sharded trainable block weights (ZeRO-3 / FSDP-style) on 2 gloo CPU ranks: each rank feeds its own
sample through a Wan block stack whose trainable weights are sharded (gathered one block ahead, gradients
reduce-scattered per block as the backward reaches it, AdamW on the shards); after three steps every
parameter equals the one of replicated data-parallel training (gradients averaged over the ranks, the
same AdamW on full tensors), and the critic-style case where a backward skips the weights (frozen for a
phase) leaves them untouched."""
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
    m = m.to(torch.bfloat16)
    m.checkpoint_blocks = 3
    m.train()
    for n, p in m.named_parameters():  # only the blocks train here
        p.requires_grad_(n.startswith("blocks."))
    return m


def _sample(rank):
    g = torch.Generator().manual_seed(100 + rank)
    return (torch.randn(1, 16, 2, 4, 4, generator=g).bfloat16(), torch.rand(1, 1, generator=g),
            torch.randn(1, 8, 32, generator=g).bfloat16())


def _adamw_reference(params, grads_per_rank, state, step, lr=1e-3, b1=0.9, b2=0.99, eps=1e-8, wd=0.01):
    """Replicated data parallel: mean of the ranks' gradients (fp32), AdamW on fp32 masters, bf16 copy."""
    bc1, bc2 = 1 - b1 ** step, 1 - b2 ** step
    for i, p in enumerate(params):
        g = sum(gr[i].float() for gr in grads_per_rank) / len(grads_per_rank)
        m, v, w = state[i]
        w.mul_(1 - lr * wd)
        m.mul_(b1).add_(g, alpha=1 - b1)
        v.mul_(b2).addcmul_(g, g, value=1 - b2)
        w.addcdiv_(m, (v / bc2).sqrt_().add_(eps), value=-lr / bc1)
        p.data.copy_(w.to(p.dtype))


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    try:
        import torch.distributed as dist
        from dmad_b200.parallel.dist import init_distributed
        from dmad_b200.parallel.fsdp import ShardedTrainableBlocks

        init_distributed(backend="gloo", timeout_s=120)
        m = _model()
        sh = ShardedTrainableBlocks(m.blocks, lr=1e-3, betas=(0.9, 0.99), eps=1e-8, weight_decay=0.01, ema=True)
        assert all(p.numel() == 0 for b in m.blocks for p in b.parameters())
        x, t, ctx = _sample(rank)
        for _ in range(3):
            out = m(x, t, ctx)
            out.float().square().mean().backward()
            sh.step(ema_beta=0.5)
            sh.zero_grad()
        # a backward with the block weights frozen for the phase: no gradient, no reduce-scatter
        for p in sh.params:
            p.requires_grad_(False)
        out = m(x.requires_grad_(True), t, ctx)
        out.float().sum().backward()
        assert not sh._pending
        full = [t_.float() for t_ in sh.full_params()]
        q.put((rank, [f.numpy() for f in full], sh.rs_count, None))
        dist.destroy_process_group()
    except Exception:  # pragma: no cover
        import traceback
        q.put((rank, None, None, traceback.format_exc()))


def test_sharded_trainable_blocks_match_replicated_dp():
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
    for rank, full, rs, err in res:
        assert err is None, err
        assert rs == 3 * 3  # one reduce-scatter per block and backward
    # replicated reference: the same model and samples, gradients of both ranks averaged
    m = _model()
    params = [p for b in m.blocks for p in b.parameters() if p.requires_grad]
    state = [(torch.zeros_like(p, dtype=torch.float32), torch.zeros_like(p, dtype=torch.float32), p.detach().float())
             for p in params]
    for step in range(1, 4):
        grads = []
        for r in range(world):
            for p in params:
                p.grad = None
            x, t, ctx_ = _sample(r)
            m(x, t, ctx_).float().square().mean().backward()
            grads.append([p.grad.detach().clone() for p in params])
        _adamw_reference(params, grads, state, step)
    for rank, full, rs, err in res:
        assert len(full) == len(params)
        for a, p in zip(full, params):
            torch.testing.assert_close(torch.from_numpy(a), p.detach().float(), rtol=0, atol=0)


def _dmad_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    try:
        import torch.distributed as dist
        from dmad_b200.distill.wan_dmad import WanDMAD, WanDMADConfig
        from dmad_b200.models.wan import WanConfig
        from dmad_b200.parallel.dist import init_distributed

        init_distributed(backend="gloo", timeout_s=120)
        net = WanConfig(dim=128, ffn_dim=256, num_heads=1, num_layers=2, text_dim=32, freq_dim=64)
        g = torch.Generator().manual_seed(30 + rank)  # each rank its own sample
        shp = (1, 16, 2, 4, 8)
        batch = {"latents": torch.randn(shp, generator=g), "real_latents": torch.randn(shp, generator=g),
                 "context": torch.randn(1, 5, 32, generator=g)}
        out = {}
        for fsdp in (False, True):
            cfg = WanDMADConfig(net=net, sn_power_iters=2, fsdp_trainable=fsdp, checkpoint_student_blocks=2,
                                checkpoint_critic_blocks=2, checkpoint_critic_blocks_student_phase=2)
            m = WanDMAD(cfg, device="cpu", dtype=torch.float32, seed=0)
            with torch.no_grad():
                for n_ in (m.net, m.net_fake_score):
                    torch.nn.init.normal_(n_.head.head.weight, std=0.05, generator=torch.Generator().manual_seed(9))
            torch.manual_seed(5 + rank)
            losses = [float(m.training_step(batch, it).get("dmad_g_loss", 0.0)) for it in range(4)]
            import copy
            # a snapshot, as the checkpointer's host copy is (the returned tensors are the live state)
            shared, per_rank = copy.deepcopy(m.state_dicts())
            out[fsdp] = (losses, shared)
            if fsdp:  # resume into a fresh sharded model: the next step matches the uninterrupted run
                torch.manual_seed(77)
                nxt = float(m.training_step(batch, 4)["dmad_g_loss"])
                m2 = WanDMAD(cfg, device="cpu", dtype=torch.float32, seed=1)
                m2.load_state_dicts(shared, per_rank)
                torch.manual_seed(77)
                nxt2 = float(m2.training_step(batch, 4)["dmad_g_loss"])
                out["resume"] = (nxt, nxt2)
        # the critic step's three backward passes are summed in another order (per pass across the ranks,
        # then over the passes, instead of over the passes first), so the weights agree to rounding
        same = max(float((out[False][1][k][n].float() - out[True][1][k][n].float()).abs().max())
                   for k in ("net", "net_fake_score") for n in out[False][1][k]) < 1e-6
        q.put((rank, out[False][0], out[True][0], same, out["resume"], None))
        dist.destroy_process_group()
    except Exception:  # pragma: no cover
        import traceback
        q.put((rank, None, None, None, None, traceback.format_exc()))


def test_wan_dmad_fsdp_trainable_matches_sharded_optimizer():
    """The Wan DMAD model with its critic and student block weights FSDP-sharded trains as with replicated
    weights and the sharded optimiser (2 ranks, different samples: the same losses, weights equal to
    rounding), and resumes from its checkpoint state."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_dmad_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=600) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    for rank, l0, l1, same, resume, err in res:
        assert err is None, err
        assert l0 == l1, (l0, l1)
        assert same
        assert resume[0] == resume[1], resume


def _hsdp_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    try:
        import copy

        import torch.distributed as dist
        from dmad_b200.distill.wan_dmad import WanDMAD, WanDMADConfig
        from dmad_b200.models.wan import WanConfig
        from dmad_b200.parallel.dist import init_distributed

        init_distributed(backend="gloo", timeout_s=120)
        net = WanConfig(dim=128, ffn_dim=256, num_heads=1, num_layers=2, text_dim=32, freq_dim=64)
        g = torch.Generator().manual_seed(60 + rank)
        shp = (1, 16, 2, 4, 8)
        batch = {"latents": torch.randn(shp, generator=g), "real_latents": torch.randn(shp, generator=g),
                 "context": torch.randn(1, 5, 32, generator=g)}
        out = {}
        for mode in ("replicated", "hsdp"):
            cfg = WanDMADConfig(net=net, sn_power_iters=2, fsdp_trainable=mode == "hsdp", fsdp_shard_size=2,
                                checkpoint_student_blocks=2, checkpoint_critic_blocks=2,
                                checkpoint_critic_blocks_student_phase=2)
            m = WanDMAD(cfg, device="cpu", dtype=torch.float32, seed=0)
            with torch.no_grad():
                for n_ in (m.net, m.net_fake_score):
                    torch.nn.init.normal_(n_.head.head.weight, std=0.05, generator=torch.Generator().manual_seed(9))
            torch.manual_seed(5 + rank)
            losses = [float(m.training_step(batch, it).get("dmad_g_loss", 0.0)) for it in range(4)]
            out[mode] = (losses, copy.deepcopy(m.state_dicts()[0]))
            if mode == "hsdp":
                sh = m.fsdp["critic"]
                out["sizes"] = (sh.world, sh.replicas)
        err = max(float((out["replicated"][1][k][n].float() - out["hsdp"][1][k][n].float()).abs().max())
                  for k in ("net", "net_fake_score") for n in out["replicated"][1][k])
        q.put((rank, out["replicated"][0], out["hsdp"][0], err, out["sizes"], None))
        dist.destroy_process_group()
    except Exception:  # pragma: no cover
        import traceback
        q.put((rank, None, None, None, None, traceback.format_exc()))


def test_wan_dmad_hsdp_matches_replicated():
    """Hybrid sharding on 4 gloo ranks: block weights sharded over pairs of ranks and replicated across
    the pairs train as plain data parallelism does (each rank its own sample)."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_hsdp_worker, args=(r, 4, port, q)) for r in range(4)]
    for p in procs:
        p.start()
    res = [q.get(timeout=900) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    for rank, l0, l1, err, sizes, e in res:
        assert e is None, e
        assert sizes == (2, 2)
        # four gradients are summed pairwise, then across the pairs, instead of in one all-reduce
        for a, b in zip(l0, l1):
            assert abs(a - b) <= 1e-5 * max(1.0, abs(a)), (l0, l1)
        assert err < 1e-5, err
