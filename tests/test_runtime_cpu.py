"""Runtime services on CPU: config system, checkpoint manager (atomic publish, pruning, async,
truncation detection), LR schedules, metrics window, iteration timeout, tar shards split by
data-parallel group, heartbeat failure detection across gloo ranks, and the training CLI with
save / resume reproducing an uninterrupted run."""
import json
import os
import socket
import time

import pytest
import torch
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


# ---------------------------------------------------------------- config
def test_config_base_env_overrides(tmp_path, monkeypatch):
    from dmad_b200.runtime.config import load_config, register_experiment, to_dataclass
    from dmad_b200.distill.wan_dmad import WanDMADConfig

    (tmp_path / "base.yaml").write_text("a: {x: 1, y: 2}\nout: ${env:DMAD_T_OUT,default_dir}/m.jsonl\nn: ${env:DMAD_T_N,3}\n")
    (tmp_path / "c.yaml").write_text("base: base.yaml\na: {y: 5}\nb: [1, 2]\n")
    monkeypatch.setenv("DMAD_T_OUT", "/tmp/o")
    register_experiment("t_exp", {"a": {"z": 9}})
    cfg = load_config(str(tmp_path / "c.yaml"), ["a.x=10", "c.d=true", "experiment=t_exp", "lr=2e-6"])
    assert cfg["a"] == {"x": 10, "y": 5, "z": 9}
    assert cfg["out"] == "/tmp/o/m.jsonl" and cfg["n"] == 3
    assert cfg["c"]["d"] is True and cfg["lr"] == 2e-6 and cfg["experiment"] == "t_exp"
    d = to_dataclass(WanDMADConfig, {"lr": 1e-5, "betas": [0.0, 0.9], "net": {"dim": 64, "num_heads": 1}})
    assert d.lr == 1e-5 and d.betas == (0.0, 0.9) and d.net.dim == 64
    with pytest.raises(KeyError):
        to_dataclass(WanDMADConfig, {"not_a_field": 1})


# ---------------------------------------------------------------- checkpoint
@pytest.mark.parametrize("async_save", [False, True])
def test_checkpoint_manager(tmp_path, async_save):
    from dmad_b200.runtime.checkpoint import CheckpointManager, find_latest_checkpoint

    m = CheckpointManager(str(tmp_path), total_limit=2, async_save=async_save)
    for it in (10, 20, 30):
        m.save(it, {"w": torch.full((4,), float(it))}, {"shard": torch.arange(3) + it}, config_text="a: 1\n")
    m.finalize()
    names = sorted(os.listdir(tmp_path))
    assert names == ["checkpoint-000000020", "checkpoint-000000030", "latest_checkpoint.txt"]
    path, it = find_latest_checkpoint(str(tmp_path))
    assert it == 30 and open(tmp_path / "latest_checkpoint.txt").read() == "checkpoint-000000030"
    shared, per_rank, manifest = m.load(path)
    assert float(shared["w"][0]) == 30.0 and int(per_rank["shard"][0]) == 30 and manifest["world_size"] == 1
    # a crashed save (left .partial) is ignored; a truncated file is detected
    os.makedirs(tmp_path / "checkpoint-000000040.partial")
    assert find_latest_checkpoint(str(tmp_path))[1] == 30
    with open(os.path.join(path, "shared.pt"), "ab") as f:
        f.write(b"x")
    with pytest.raises(RuntimeError, match="truncated"):
        m.load(path)


def test_lr_schedule_and_metrics(tmp_path):
    from dmad_b200.runtime.logging import MetricsWriter
    from dmad_b200.runtime.lr import LRSchedule, lr_factor

    class O:
        lr = 1.0

    s = LRSchedule(O(), "linear", warmup=2, total=10)
    lrs = [s.opt.lr]
    for _ in range(10):
        s.step()
        lrs.append(s.opt.lr)
    assert lrs[0] == 0.5 and lrs[1] == 1.0 and lrs[-1] == 0.0
    assert abs(lr_factor("cosine", 6, 2, 10) - 0.5) < 1e-9
    w = MetricsWriter(str(tmp_path / "m.jsonl"), every=2)
    w.add({"dmad_g_loss": torch.tensor(1.0), "x": 3})
    w.add({"dmad_g_loss": torch.tensor(3.0), "x": 5, "vec": torch.ones(2)})
    rec = w.flush(2)
    assert rec["dmad_g_loss"] == 2.0 and rec["x"] == 4.0 and "vec" not in rec
    assert json.loads(open(tmp_path / "m.jsonl").read())["iteration"] == 2


def test_iteration_timeout():
    from dmad_b200.runtime.watchdog import IterationTimeout

    with pytest.raises(TimeoutError):
        with IterationTimeout(1):
            time.sleep(3)
    with IterationTimeout(2) as t:  # kicked in time: no error
        for _ in range(3):
            time.sleep(0.5)
            t.kick()


def test_tar_shards_split_by_dp_group(tmp_path):
    from dmad_b200.data import TarShardDataset, write_shard

    for s in range(4):
        write_shard(str(tmp_path / f"s{s}.tar"), [
            {"__key__": f"k{s}_{i}", "latent.pt": torch.full((2, 3), float(10 * s + i)),
             "embed.pt": torch.zeros(4, 5), "prompt.txt": f"p{s}{i}", "real_latent.pt": torch.ones(2, 3)}
            for i in range(3)])
    seen = {}
    for rank in range(4):  # world 4, cp 2 -> dp groups {0,1}, {2,3}
        ds = TarShardDataset(str(tmp_path / "*.tar"), batch_size=2, rank=rank, world=4, cp_size=2,
                             shuffle_buffer=1, epochs=1, partial=True)
        vals = []
        for b in ds:
            assert b["latents"].shape[1:] == (2, 3) and isinstance(b["prompts"], list)
            assert b["t5_text_embeddings"].shape[1:] == (4, 5) and "real_latents" in b
            vals += b["latents"][:, 0, 0].tolist()
        seen[rank] = sorted(vals)
    assert seen[0] == seen[1] and seen[2] == seen[3]
    assert sorted(seen[0] + seen[2]) == sorted(float(10 * s + i) for s in range(4) for i in range(3))


# ---------------------------------------------------------------- heartbeat failure detection
def _hb_worker(rank, world, port, q):
    import torch.distributed as dist
    from dmad_b200.runtime.watchdog import Heartbeat, PeerFailure

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    hb = Heartbeat(rank, world, interval_s=0.2).start()
    time.sleep(0.6)
    ok_before = not hb.stale_peers(1.0)
    if rank == world - 1:
        hb.stop()  # this rank "hangs": it stops beating and never joins another collective
        time.sleep(4.0)
        q.put((rank, ok_before, None))
        return
    detected = None
    t0 = time.time()
    while time.time() - t0 < 10:
        try:
            hb.check(1.0)
        except PeerFailure as e:
            detected = e.ranks
            break
        time.sleep(0.2)
    hb.stop()
    q.put((rank, ok_before, detected))


def test_heartbeat_detects_dead_rank():
    world = 3
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_hb_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    for rank, ok_before, detected in res:
        assert ok_before
        if rank < world - 1:
            assert detected == [world - 1]


# ---------------------------------------------------------------- training CLI: save / resume
_TINY = ["model.net={dim: 128, ffn_dim: 256, num_heads: 1, num_layers: 2, text_dim: 32, freq_dim: 64}",
         "model.distill.lr=1.0e-3", "model.distill.critic_lr=1.0e-3", "model.distill.sn_power_iters=2",
         "data.latent_shape=[16, 2, 4, 4]", "data.text_shape=[8, 32]", "data.fixed=false",
         "training.log_every=2", "training.timeout_s=300", "training.heartbeat_s=0", "training.async_save=false"]


def _train_worker(rank, world, port, out_dir, stages, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    try:
        import torch.distributed as dist
        from dmad_b200.runtime.config import load_config
        from dmad_b200.train.trainer import DistillTrainer

        cfg_path = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "configs",
                                "wan_1p3b_dmad.yaml")
        final = None
        for max_iters, resume in stages:
            cfg = load_config(cfg_path, _TINY + [f"training.output_dir={out_dir}", f"training.max_iters={max_iters}",
                                                 "training.save_every=2", f"training.auto_resume={resume}"])
            tr = DistillTrainer(cfg)
            tr.train()
            final = torch.cat([p.detach().float().reshape(-1) for p in tr.model.net.parameters()])
            if dist.is_initialized():
                dist.barrier()
        q.put((rank, final.numpy(), None))
        dist.destroy_process_group()
    except Exception:  # pragma: no cover
        import traceback
        q.put((rank, None, traceback.format_exc()))


def _run_train(tmp_path, name, stages, world=2):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    out = str(tmp_path / name)
    procs = [ctx.Process(target=_train_worker, args=(r, world, port, out, stages, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=600) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    for _, _, err in res:
        assert err is None, err
    return out, res


def test_train_cli_resume_matches_uninterrupted(tmp_path):
    out_a, res_a = _run_train(tmp_path, "a", [(6, False)])
    out_b, res_b = _run_train(tmp_path, "b", [(4, False), (6, True)])
    assert sorted(os.listdir(out_b))[:2] == ["checkpoint-000000004", "checkpoint-000000006"] or \
        "checkpoint-000000006" in os.listdir(out_b)
    lines = [json.loads(x) for x in open(os.path.join(out_a, "metrics.jsonl"))]
    assert lines[-1]["iteration"] == 6 and "dmad_g_loss" in lines[0]
    for (ra, wa, _), (rb, wb, _) in zip(res_a, res_b):
        assert torch.equal(torch.from_numpy(wa), torch.from_numpy(wb)), "resumed run diverged"


def test_export_release_folds_sn_and_uses_ema(tmp_path):
    """Train 4 tiny iterations in-process, export the EMA student with SN folded, and check the
    plain (no SN, no LoRA) network reproduces the student's EMA forward."""
    from dmad_b200.models.wan import WanConfig, WanModel
    from dmad_b200.runtime.config import load_config
    from dmad_b200.tools.export_release import build_student, export
    from dmad_b200.train.trainer import DistillTrainer

    cfg_path = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "configs",
                            "wan_1p3b_dmad.yaml")
    cfg = load_config(cfg_path, _TINY + [f"training.output_dir={tmp_path}", "training.max_iters=4",
                                         "training.save_every=4", "model.distill.ema_rate=0.5"])
    tr = DistillTrainer(cfg)
    tr.train()
    ck = os.path.join(str(tmp_path), "checkpoint-000000004")
    sd = export(ck, str(tmp_path / "release.pth"), use_ema=True, dtype=torch.float32)
    assert all(k.startswith("net.") for k in sd) and not any("sn_" in k for k in sd)
    plain = WanModel(WanConfig(dim=128, ffn_dim=256, num_heads=1, num_layers=2, text_dim=32, freq_dim=64))
    plain.load_state_dict({k[4:]: v for k, v in sd.items()})
    # reference: the trained student with its EMA weights, SN applied from the stored vectors
    stud = build_student(cfg)
    stud.load_state_dict(tr.model.net.state_dict())
    ema = dict(zip([n for n, p in tr.model.net.named_parameters() if p.requires_grad], tr.model.ema_weights()))
    with torch.no_grad():
        for n, p in stud.named_parameters():
            p.copy_(ema[n])
    stud.eval()
    plain.eval()
    g = torch.Generator().manual_seed(0)
    x, t, ctx = torch.randn(1, 16, 2, 4, 4, generator=g), torch.rand(1, 1, generator=g), torch.randn(1, 8, 32, generator=g)
    with torch.no_grad():
        a, b = stud(x, t, ctx), plain(x, t, ctx)
    assert (a - b).abs().max().item() < 1e-3 * max(1.0, a.abs().max().item())
    assert not torch.equal(ema[next(iter(ema))], tr.model.net.state_dict()[next(iter(ema))])


def test_train_cli_edm_family(tmp_path):
    """The CLI trains the EDM config-1 family (own synthetic batches) and resumes it."""
    from dmad_b200.cli.train import main

    cfg = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "configs",
                       "edm_imagenet64_dmad.yaml")
    out = str(tmp_path / "edm")
    main(["--config", cfg, f"training.output_dir={out}", "training.max_iters=2", "training.save_every=1",
          "training.log_every=1"])
    assert "checkpoint-000000002" in os.listdir(out)
    main(["--config", cfg, f"training.output_dir={out}", "training.max_iters=3", "training.save_every=1",
          "training.log_every=1"])
    assert "checkpoint-000000003" in os.listdir(out)
    lines = [json.loads(x) for x in open(os.path.join(out, "metrics.jsonl"))]
    assert lines[-1]["iteration"] == 3 and "generator_loss" in lines[-1]


def test_elastic_resume_on_another_world_size(tmp_path):
    """A 2-rank run's checkpoint (per-rank optimiser shards) resumes in one process only with
    ``training.elastic_resume``; the shards are resharded and training continues."""
    from dmad_b200.runtime.config import load_config
    from dmad_b200.train.trainer import DistillTrainer

    out, _ = _run_train(tmp_path, "c", [(4, False)])
    cfg_path = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "configs",
                            "wan_1p3b_dmad.yaml")
    base = _TINY + [f"training.output_dir={out}", "training.max_iters=6", "training.save_every=0",
                    "training.auto_resume=true"]
    with pytest.raises(RuntimeError, match="world_size"):
        DistillTrainer(load_config(cfg_path, base)).train()
    tr = DistillTrainer(load_config(cfg_path, base + ["training.elastic_resume=true"]))
    tr.train()
    assert tr.iteration == 6
    assert all(torch.isfinite(p).all() for p in tr.model.net.parameters())


def test_every_n_draw_sample_and_ema_scope(tmp_path):
    """``training.sample_every``: 1-, 2- and 4-step samples of the batch saved as latents; with
    ``sample_ema`` the student runs with its EMA weights and gets its own weights back afterwards."""
    from dmad_b200.runtime.config import load_config
    from dmad_b200.train.trainer import DistillTrainer

    cfg_path = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "configs",
                            "wan_1p3b_dmad.yaml")
    cfg = load_config(cfg_path, _TINY + [f"training.output_dir={tmp_path}", "training.max_iters=4",
                                         "training.save_every=100", "model.distill.ema_rate=0.5",
                                         "training.sample_every=2", "training.sample_ema=true"])
    tr = DistillTrainer(cfg)
    tr.train()
    files = sorted(os.listdir(tmp_path / "samples"))
    assert files == ["iter_000000002_ema_rank000.pt", "iter_000000004_ema_rank000.pt"]
    rec = torch.load(tmp_path / "samples" / files[-1])
    assert set(rec) >= {"steps_1", "steps_2", "steps_4"} and rec["steps_4"].shape == (1, 16, 2, 4, 4)
    assert all(torch.isfinite(rec[k]).all() for k in ("steps_1", "steps_2", "steps_4"))
    m = tr.model
    before = [p.detach().clone() for p in m._student_params]
    ema = m.ema_weights()
    with m.ema_scope():
        assert all(torch.equal(p, e.to(p.dtype).view_as(p)) for p, e in zip(m._student_params, ema))
    assert all(torch.equal(p, b) for p, b in zip(m._student_params, before))
    assert not all(torch.equal(b, e.to(b.dtype).view_as(b)) for b, e in zip(before, ema))
