"""H3 DMAD with its block weights sharded over 2 gloo CPU ranks (the LoRA student's frozen base, the
critic's frozen first blocks, and, in full-critic mode, the critic's trainable blocks FSDP-style) trains
as the unsharded model does: the same losses and the same weights to rounding after two iterations."""
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


def _run(shard):
    from dmad_b200.distill.h3_dmad import H3DMAD, H3DMADConfig
    from dmad_b200.models.h3 import H3Config

    cfg = H3DMADConfig(model=H3Config(dim=64, num_heads=1, ffn_dim=96, num_layers=4, refiner_layers=1, text_dim=16,
                                      time_embed_dim=32), height=64, width=64, num_frames=22, student_lora_rank=4,
                       text_tokens=4, fake_train_type="full", critic_freeze_blocks=2, shard_weights=shard)
    m = H3DMAD(cfg, "cpu", dtype=torch.float32, seed=0)
    torch.manual_seed(11)
    losses = []
    for _ in range(2):
        out = m.train_iteration()
        losses += [out["student"]["loss"], out["critic0"]["gan_d"]]
    if shard:
        crit = [t.float() for t in m.fake_fsdp.full_params()]
    else:
        crit = [p.detach().float().clone() for b in list(m.fake.transformer_blocks)[2:] for p in b.parameters()
                if p.requires_grad]
    lora = [p.detach().float().clone() for p in m.s_params]
    return losses, crit, lora


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    try:
        import torch.distributed as dist
        from dmad_b200.parallel.dist import init_distributed

        init_distributed(backend="gloo", timeout_s=120)
        ref = _run(False)
        sh = _run(True)
        crit_err = max(float((a - b).abs().max()) for a, b in zip(ref[1], sh[1]))
        lora_err = max(float((a - b).abs().max()) for a, b in zip(ref[2], sh[2]))
        q.put((rank, ref[0], sh[0], crit_err, lora_err, None))
        dist.destroy_process_group()
    except Exception:  # pragma: no cover
        import traceback
        q.put((rank, None, None, None, None, traceback.format_exc()))


def test_h3_dmad_sharded_matches_unsharded():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=600) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    for rank, l_ref, l_sh, crit_err, lora_err, err in res:
        assert err is None, err
        for a, b in zip(l_ref, l_sh):
            assert abs(a - b) <= 1e-5 * max(1.0, abs(a)), (l_ref, l_sh)
        assert crit_err < 1e-5 and lora_err < 1e-5, (crit_err, lora_err)
