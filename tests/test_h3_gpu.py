"""H3-shaped model on the GPU: kernels vs the CPU math, and the low-VRAM streamed rollout is
bit-identical to the resident rollout."""
import copy

import pytest
import torch

pytestmark = pytest.mark.gpu


def _tiny():
    from dmad_b200.models.h3 import H3Config, H3Model
    torch.manual_seed(0)
    cfg = H3Config(dim=256, num_heads=2, ffn_dim=512, num_layers=4, text_dim=128, time_embed_dim=128)
    m = H3Model(cfg)
    for p in m.parameters():
        p.data.normal_(0, 0.03)
    return cfg, m


def _inputs(device):
    from dmad_b200.inference.h3 import H3Geometry, build_packed_sequence, latent_shape_of
    geo = H3Geometry()
    shape = latent_shape_of(128, 192, 22, geo)
    lay = build_packed_sequence(torch.ones(20, dtype=torch.long), shape["latent_frames"], shape["latent_height"],
                                shape["latent_width"], shape["audio_latents"])
    return geo, shape, lay


def test_h3_forward_matches_cpu():
    from dmad_b200.inference.h3 import build_row_timesteps
    cfg, m = _tiny()
    geo, shape, lay = _inputs("cpu")
    ts, ti = build_row_timesteps(lay, torch.tensor(0.7), torch.tensor(0.4))
    g = torch.Generator().manual_seed(1)
    v = torch.randn(shape["video_tokens"], generator=g)
    a = torch.randn(shape["audio_tokens"], generator=g)
    pe = torch.randn(1, 20, 128, generator=g)
    kw = dict(timestep=ts, timestep_indices=ti, token_tags=lay.token_tags, position_ids=lay.position_ids,
              video_indices=lay.video_indices, audio_indices=lay.audio_indices, text_indices=lay.text_indices)
    ref = m(v, a, pe, **kw)
    mg = copy.deepcopy(m).cuda().to(torch.bfloat16)
    kwg = {k: x.cuda() for k, x in kw.items()}
    out = mg(v.cuda(), a.cuda(), pe.cuda(), **kwg)
    for o, r in zip(out, ref):
        assert ((o.float().cpu() - r).norm() / r.norm()).item() < 5e-2


def test_lowmem_streamed_is_bit_identical():
    from dmad_b200.inference.h3 import build_row_timesteps, rollout, sigma_grid
    from dmad_b200.inference.lowmem import LowMemH3
    cfg, m = _tiny()
    m = m.to(torch.bfloat16).eval().requires_grad_(False)
    geo, shape, lay = _inputs("cuda")
    vs, as_ = sigma_grid(4, 12.0), sigma_grid(4, 2.0)
    pe = torch.randn(1, 20, 128).to(torch.bfloat16)
    resident = copy.deepcopy(m).cuda()
    ref = rollout(resident, pe.cuda(), lay, shape, geo, vs, as_, 7, torch.device("cuda"))
    ts = [build_row_timesteps(lay, vs[s], as_[s])[0] for s in range(4)]
    lm = LowMemH3(copy.deepcopy(m), torch.device("cuda"), ts)
    lm.precompute_text([pe])
    out = rollout(lm.model, pe.cuda(), lay, shape, geo, vs, as_, 7, torch.device("cuda"),
                  text_features=lm.text_features(pe), adaln_tables_per_step=lm.tables)
    lm.close()
    assert torch.equal(out[0], ref[0]) and torch.equal(out[1], ref[1])


@pytest.mark.parametrize("layers", [3, 4])
def test_lowmem_streamed_from_shards_is_bit_identical(tmp_path, layers):
    """Blocks streamed from memory-mapped safetensors through pinned staging buffers (odd and even block
    counts, so the slot rotation wraps both ways) give the resident rollout bit for bit."""
    import json

    from safetensors.torch import save_file

    from dmad_b200.inference.h3 import build_row_timesteps, rollout, sigma_grid
    from dmad_b200.inference.lowmem import LowMemH3, build_streamed_h3
    from dmad_b200.models.h3 import H3Config, H3Model
    torch.manual_seed(0)
    m = H3Model(H3Config(dim=256, num_heads=2, ffn_dim=512, num_layers=layers, text_dim=128, time_embed_dim=128))
    for p in m.parameters():
        p.data.normal_(0, 0.03)
    m = m.to(torch.bfloat16).eval().requires_grad_(False)
    tf = tmp_path / "transformer"
    tf.mkdir()
    json.dump({"num_attention_heads": 2, "attention_head_dim": 128, "ffn_dim": 512, "num_layers": layers,
               "text_embed_dim": 128, "time_embed_dim": 128}, open(tf / "config.json", "w"))
    save_file({k: v.contiguous() for k, v in m.state_dict().items()}, str(tf / "model.safetensors"))
    geo, shape, lay = _inputs("cuda")
    vs, as_ = sigma_grid(4, 12.0), sigma_grid(4, 2.0)
    pe = torch.randn(1, 20, 128).to(torch.bfloat16)
    ref = rollout(copy.deepcopy(m).cuda(), pe.cuda(), lay, shape, geo, vs, as_, 7, torch.device("cuda"))
    ts = [build_row_timesteps(lay, vs[s], as_[s])[0] for s in range(4)]
    model, source = build_streamed_h3(tmp_path, torch.device("cuda"))
    lm = LowMemH3(model, torch.device("cuda"), ts, source=source, cache_in_ram=False)
    lm.precompute_text([pe])
    out = rollout(lm.model, pe.cuda(), lay, shape, geo, vs, as_, 7, torch.device("cuda"),
                  text_features=lm.text_features(pe), adaln_tables_per_step=lm.tables)
    lm.close()
    assert torch.equal(out[0], ref[0]) and torch.equal(out[1], ref[1])


def _h3_train_cfg(shard=False, full=False):
    from dmad_b200.distill.h3_dmad import H3DMADConfig
    from dmad_b200.models.h3 import H3Config
    return H3DMADConfig(model=H3Config(dim=256, num_heads=2, ffn_dim=512, num_layers=4, refiner_layers=1, text_dim=128,
                                       time_embed_dim=128), height=128, width=192, num_frames=22, student_lora_rank=16,
                        text_tokens=20, fake_train_type="full" if full else "lora", critic_freeze_blocks=2,
                        shard_weights=shard)


def _nonzero_outputs(m):
    """The H3 output projections start at zero (as in the reference), which keeps every gradient upstream
    of them at zero on a random-init model; give them small weights so the test sees the updates."""
    with torch.no_grad():
        for net in (m.student, m.fake):
            for lin in (net.proj_out, net.audio_proj_out):
                lin.weight.normal_(0.0, 0.02, generator=torch.Generator(device=lin.weight.device).manual_seed(3))


@pytest.mark.parametrize("full", [False, True])
def test_h3_dmad_training_on_gpu(full):
    """Two H3 DMAD iterations (student and critic stages, LoRA or full critic) run on the GPU kernels with
    finite losses, and the trainable weights move."""
    from dmad_b200 import ops
    from dmad_b200.distill.h3_dmad import H3DMAD

    m = H3DMAD(_h3_train_cfg(full=full), "cuda", dtype=torch.bfloat16)
    _nonzero_outputs(m)
    before = [p.detach().clone() for p in m.s_params]
    fbefore = [p.detach().clone() for p in m.f_params]
    for _ in range(2):
        out = m.train_iteration()
        for stage in out.values():
            assert all(torch.isfinite(torch.tensor(float(v))) for v in stage.values()), out
    torch.cuda.synchronize()
    ops.check_device_status()
    assert any(not torch.equal(a, b) for a, b in zip(before, m.s_params))
    assert any(not torch.equal(a, b) for a, b in zip(fbefore, m.f_params))


def _h3_shard_worker(rank, world, port, q):
    import os
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank), NCCL_NVLS_ENABLE="0")
    try:
        import torch.distributed as dist
        from dmad_b200.distill.h3_dmad import H3DMAD
        from dmad_b200.ops import check_device_status
        from dmad_b200.parallel.dist import init_distributed

        _, _, dev = init_distributed(timeout_s=60)
        m = H3DMAD(_h3_train_cfg(shard=True, full=True), dev, dtype=torch.bfloat16)
        _nonzero_outputs(m)
        losses = []
        for _ in range(2):
            out = m.train_iteration()
            losses.append(out["student"]["loss"])
        crit = torch.cat([t.float().reshape(-1) for t in m.fake_fsdp.full_params()])
        torch.cuda.synchronize()
        check_device_status()
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, losses, float(crit.norm()), None))
    except Exception:  # pragma: no cover
        import traceback
        q.put((rank, None, None, traceback.format_exc()))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_h3_dmad_sharded_training_two_gpus():
    """H3 DMAD with the block weights sharded over 2 GPUs (frozen bases, FSDP-sharded trainable critic
    blocks): both ranks run two iterations and end with the same critic weights."""
    import socket

    import torch.multiprocessing as mp
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_h3_shard_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    for rank, losses, norm, err in res:
        assert err is None, err
        assert all(torch.isfinite(torch.tensor(v)) for v in losses)
    assert res[0][2] == res[1][2]
