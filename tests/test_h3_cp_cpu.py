"""H3 packed-sequence context parallelism on 2 gloo CPU ranks: the velocity of the sharded model
(sequence padded at its end to a multiple of cp, padded keys excluded) equals the unsharded one."""
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


def _setup():
    from dmad_b200.inference.h3 import H3Geometry, build_packed_sequence, build_row_timesteps
    from dmad_b200.models.h3 import H3Config, H3Model

    torch.manual_seed(0)
    cfg = H3Config(dim=128, num_heads=2, ffn_dim=192, num_layers=2, refiner_layers=1, text_dim=32,
                   time_embed_dim=64, in_channels=24, audio_in_channels=32)
    m = H3Model(cfg).eval()
    geo = H3Geometry()
    lay = build_packed_sequence(torch.ones(5, dtype=torch.long), 3, 2, 4, 4)  # odd total length
    ts, ti = build_row_timesteps(lay, torch.tensor(0.7), torch.tensor(0.4))
    g = torch.Generator().manual_seed(1)
    nv = len(lay.video_indices)
    na = len(lay.audio_indices)
    pin = cfg.in_channels * 4
    kw = dict(hidden_states=torch.randn(1, nv, pin, generator=g), audio_hidden_states=torch.randn(1, na, 32, generator=g),
              encoder_hidden_states=torch.randn(1, 5, 32, generator=g), timestep=ts, timestep_indices=ti,
              token_tags=lay.token_tags, position_ids=lay.position_ids, video_indices=lay.video_indices,
              audio_indices=lay.audio_indices, text_indices=lay.text_indices)
    return m, kw, lay.sequence_length


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    try:
        import torch.distributed as dist
        from dmad_b200.parallel.cp import ContextParallel
        from dmad_b200.parallel.dist import init_distributed

        init_distributed(backend="gloo", timeout_s=120)
        m, kw, L = _setup()
        m.enable_context_parallel(ContextParallel(impl="nccl"))
        with torch.no_grad():
            v, a = m(**kw)
            feats = m(**kw, stop_after_block=1)
        q.put((rank, v.numpy(), a.numpy(), feats.numpy(), L, None))
        dist.destroy_process_group()
    except Exception:  # pragma: no cover
        import traceback
        q.put((rank, None, None, None, None, traceback.format_exc()))


def test_h3_cp_matches_unsharded():
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
    m, kw, L = _setup()
    with torch.no_grad():
        v, a = m(**kw)
        feats = m(**kw, stop_after_block=1)
    for rank, vv, aa, ff, LL, err in res:
        assert err is None, err
        assert LL % world == 1  # the packed length needs padding
        torch.testing.assert_close(torch.from_numpy(vv), v, rtol=1e-4, atol=1e-5)
        torch.testing.assert_close(torch.from_numpy(aa), a, rtol=1e-4, atol=1e-5)
        torch.testing.assert_close(torch.from_numpy(ff), feats, rtol=1e-4, atol=1e-5)
