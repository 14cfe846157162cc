"""The config-3 training combination on 2 gloo CPU ranks: a LoRA student whose frozen base and the
frozen teacher are sharded over the ranks, Ulysses context parallelism over both ranks, the sCM
consistency term (forward-mode JVP of the student) and the DMAD critic, as bench.py runs it for the
Wan-14B shape.  One generator and one critic iteration must run, give finite losses that agree on
both ranks (they share one sample), and update the trainable weights identically on both."""
import os
import socket

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
        from dmad_b200.parallel.cp import make_context_parallel
        from dmad_b200.parallel.dist import init_distributed
        from dmad_b200.train.trainer import make_cp_group

        init_distributed(backend="gloo", timeout_s=120)
        net = WanConfig(dim=256, ffn_dim=512, num_heads=2, num_layers=2, text_dim=32, freq_dim=64)
        cfg = WanDMADConfig(net=net, sn_power_iters=2, student_lora_rank=4, shard_frozen=True,
                            checkpoint_student_blocks=2, checkpoint_critic_blocks=2,
                            checkpoint_critic_blocks_student_phase=2, loss_scale=100.0, teacher_guidance=5.0)
        m = WanDMAD(cfg, device="cpu", dtype=torch.float32, seed=0)
        with torch.no_grad():  # the Wan head starts at zero (as the reference's); no gradient reaches the
            for n_ in (m.net, m.net_fake_score):  # blocks through it until it is non-zero
                torch.nn.init.normal_(n_.head.head.weight, std=0.05, generator=torch.Generator().manual_seed(9))
        cpc = make_context_parallel(make_cp_group(2), impl="nccl")
        for n in m.context_parallel_nets():
            n.enable_context_parallel(cpc)
        g = torch.Generator().manual_seed(3)  # the same sample on both ranks (one CP group)
        shp = (1, 16, 2, 4, 8)
        batch = {"latents": torch.randn(shp, generator=g), "real_latents": torch.randn(shp, generator=g),
                 "context": torch.randn(1, 5, 32, generator=g)}
        torch.manual_seed(100)  # identical draws on both ranks
        lora_before = torch.cat([p.detach().reshape(-1).clone() for n_, p in m.net.named_parameters()
                                 if p.requires_grad])
        o1 = m.training_step(batch, 0)
        o2 = m.training_step(batch, 1)
        lora_after = torch.cat([p.detach().reshape(-1) for n_, p in m.net.named_parameters() if p.requires_grad])
        # the 4-step generation bench.py times, through the sharded student under CP
        gen = m.generate(batch["context"], shp, num_steps=4, generator=torch.Generator().manual_seed(5))
        vals = torch.tensor([float(o1["dmad_g_loss"]), float(o1.get("scm_loss", o1.get("loss_scm", 0.0))),
                             float(o2["dmad_d_loss"]), float((lora_after - lora_before).abs().sum()),
                             float(gen.float().abs().mean())])
        q.put((rank, vals.tolist(), lora_after.sum().item(), sorted(o1.keys())))
        dist.destroy_process_group()
    except Exception as e:  # pragma: no cover - reported to the parent
        import traceback
        q.put((rank, repr(e) + traceback.format_exc(), None, None))


def test_lora_cp_scm_dmad_step_on_two_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(2):
        r, vals, s, keys = q.get(timeout=600)
        res[r] = (vals, s, keys)
    for p in procs:
        p.join(timeout=60)
    for r in range(2):
        assert isinstance(res[r][0], list), res[r][0]
    v0, v1 = res[0][0], res[1][0]
    assert all(abs(x) < float("inf") and x == x for x in v0), v0
    assert v0[3] > 0, "the LoRA weights did not move"
    for a, b in zip(v0, v1):
        assert abs(a - b) <= 1e-4 * max(1.0, abs(a)), (v0, v1)
    assert abs(res[0][1] - res[1][1]) <= 1e-5 * max(1.0, abs(res[0][1]))
