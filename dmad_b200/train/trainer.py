"""The distillation training loop (Wan DMAD / rCM; one process per GPU).

Parity: the Wan distillation trainer (train/wan/rcm/trainers/trainer_distillation.py:42-319:
data -> ``training_step`` with student / critic phases -> per-phase optimiser and scheduler ->
EMA -> checkpoint every ``save_iter`` -> SIGALRM timeout re-armed per iteration -> profiler
step) and the H3 DMD trainer's resume / pruning / world-size validation
(train/h3/lightx2v_train/trainers/dmd/trainer.py:118-265).

Config sections (YAML, see ``configs/``):

    model:     {family: wan_dmad, net: wan2.1-1.3b | wan2.1-14b | {dim: ..}, distill: {WanDMADConfig fields}}
    data:      {kind: synthetic | shards, pattern, batch_size, latent_shape, text_shape, shuffle_buffer}
    parallel:  {cp: 1, cp_impl: fused | nccl, dp_optimizer: sharded | replicated}
    training:  {max_iters, output_dir, save_every, save_total_limit, auto_resume, async_save, seed,
                lr_schedule, lr_warmup, timeout_s, log_every, heartbeat_s, heartbeat_max_age_s}
    logging:   {metrics_file, log_file}
    profiling: {enabled, wait, warmup, active, dir, memory_snapshot}
"""
from __future__ import annotations

import datetime
import os

import torch
import torch.distributed as dist

from ..parallel.dist import barrier, get_rank, get_world_size, init_distributed, is_distributed
from ..runtime import callbacks as cbs
from ..runtime.checkpoint import CheckpointManager
from ..runtime.config import get_dotted, save_config, to_dataclass
from ..runtime.logging import MetricsWriter, get_logger
from ..runtime.lr import LRSchedule
from ..runtime.profiling import maybe_memory_snapshot, maybe_profile
from ..runtime.watchdog import Heartbeat, IterationTimeout
from .registry import build_model


def make_cp_group(cp: int):
    """Split the world into consecutive groups of ``cp`` ranks; returns this rank's group."""
    world, rank = get_world_size(), get_rank()
    if cp <= 1:
        return None
    if world % cp:
        raise ValueError(f"world size {world} is not divisible by cp={cp}")
    mine = None
    for g in range(world // cp):
        ranks = list(range(g * cp, (g + 1) * cp))
        grp = dist.new_group(ranks)
        if rank in ranks:
            mine = grp
    return mine


class DistillTrainer:
    def __init__(self, cfg: dict, dryrun: bool = False):
        self.cfg = cfg
        tr = cfg.get("training", {})
        self.max_iters = int(tr.get("max_iters", 100))
        self.output_dir = tr.get("output_dir", "outputs/run")
        self.save_every = int(tr.get("save_every", 0) or 0)
        self.log_every = int(tr.get("log_every", 10))
        self.rank, self.world, self.device = init_distributed(timeout_s=float(tr.get("pg_timeout_s", 1800)))
        seed = int(tr.get("seed", 0))
        self.log = get_logger("dmad_b200.train", log_file=get_dotted(cfg, "logging.log_file"))
        cp = int(get_dotted(cfg, "parallel.cp", 1) or 1)
        self.cp_size = cp
        self.dp_rank = self.rank // cp
        self.model = build_model(cfg, self.device, seed=seed)
        if cp > 1:
            from ..parallel.cp import make_context_parallel
            grp = make_cp_group(cp)
            self.cp = make_context_parallel(grp, impl=get_dotted(cfg, "parallel.cp_impl", "fused"), device=self.device,
                                            ulysses_size=get_dotted(cfg, "parallel.ulysses_size", None))
            for net in self.model.context_parallel_nets():
                net.enable_context_parallel(self.cp)
        else:
            self.cp = None
        # every rank of a CP group draws the same random numbers (one sample per group)
        torch.manual_seed(seed + 7919 * self.dp_rank)
        self.data = None  # built at train() time, after a resume has set the start iteration
        sched = tr.get("lr_schedule", "constant")
        warm = int(tr.get("lr_warmup", 0))
        cycles = tr.get("lr_cycles")  # lambda_* schedules: warm_up_steps / cycle_lengths / f_start / f_max / f_min
        self.schedules = {name: LRSchedule(opt, sched, warm, self.max_iters, cycles=cycles) for name, opt in
                          self.model.optimizers().items()}
        self.ckpt = CheckpointManager(self.output_dir, tr.get("save_total_limit"), bool(tr.get("async_save", False)))
        self.metrics = MetricsWriter(get_dotted(cfg, "logging.metrics_file", os.path.join(self.output_dir,
                                                                                          "metrics.jsonl")),
                                     every=self.log_every)
        self.callbacks = [cbs.IterSpeed(self.log_every), cbs.DataLoadingSpeed(), cbs.ForceFiniteLoss(),
                          cbs.DeviceMonitor(max(self.log_every, 50))]
        hb = float(tr.get("heartbeat_s", 0) or 0)
        if hb > 0 and self.world > 1:
            self.callbacks.append(cbs.HeartBeatCallback(Heartbeat(self.rank, self.world, hb),
                                                        float(tr.get("heartbeat_max_age_s", 10 * hb))))
        if int(tr.get("sample_every", 0) or 0) > 0:
            self.callbacks.append(cbs.EveryNDrawSample(self.output_dir, int(tr["sample_every"]),
                                                       int(tr.get("sample_steps", 4)), bool(tr.get("sample_ema", False)),
                                                       int(tr.get("sample_ranks", 1))))
        self.timeout = IterationTimeout(tr.get("timeout_s"))
        self.dryrun = dryrun
        self.last_batch = None
        self.iteration = 0

    # ------------------------------------------------------------------ data
    def _build_data(self, d: dict):
        from ..data import DevicePrefetcher, SyntheticWanData, TarShardDataset

        kind = d.get("kind", "synthetic")
        bs = int(d.get("batch_size", 1))
        if kind in ("internal", "h3_pool"):  # the model draws its own batches (H3 pool, EDM / SDXL synthetic)
            import itertools
            return itertools.repeat(None)
        if kind == "synthetic":
            src = SyntheticWanData(tuple(d.get("latent_shape", (16, 21, 60, 104))),
                                   tuple(d.get("text_shape", (512, 4096))), bs, self.dp_rank,
                                   seed=int(d.get("seed", 1234)), fixed=bool(d.get("fixed", False)),
                                   start_iteration=self.iteration)
            return DevicePrefetcher(src, self.device)
        if kind == "shards":
            ds = TarShardDataset(d["pattern"], bs, self.rank, self.world, self.cp_size,
                                 int(d.get("shuffle_buffer", 1000)), int(d.get("seed", 0)))
            loader = torch.utils.data.DataLoader(ds, batch_size=None, num_workers=int(d.get("num_workers", 2)),
                                                 pin_memory=torch.cuda.is_available())
            return DevicePrefetcher(loader, self.device, rename={"t5_text_embeddings": "context"})
        raise ValueError(f"unknown data kind {kind!r}")

    # ------------------------------------------------------------------ checkpoint
    def save(self):
        shared, per_rank = self.model.state_dicts()
        per_rank = dict(per_rank or {})
        per_rank["rng"] = {"cpu": torch.get_rng_state(),
                           "cuda": torch.cuda.get_rng_state(self.device) if self.device.type == "cuda" else None}
        shared["trainer"] = {"iteration": self.iteration, "world_size": self.world,
                             "schedules": {k: s.state_dict() for k, s in self.schedules.items()}}
        import yaml

        text = yaml.safe_dump(self.cfg, sort_keys=False)
        self.ckpt.save(self.iteration, shared, per_rank, config_text=text)
        export = getattr(self.model, "export_artifacts", None)
        if export is not None and self.rank == 0:
            from ..runtime.checkpoint import checkpoint_name
            self.ckpt.finalize()
            export(os.path.join(self.output_dir, checkpoint_name(self.iteration)))
        self.log.info("saved checkpoint iteration=%d in %s", self.iteration, self.output_dir)

    def maybe_resume(self) -> int:
        tr = self.cfg.get("training", {})
        path = tr.get("resume_from")
        if path is None and tr.get("auto_resume", False):
            path, _ = self.ckpt.latest()
        if path is None:
            return 0
        elastic = bool(tr.get("elastic_resume", False))
        shared, per_rank, manifest = self.ckpt.load(path, elastic=elastic)
        old_world = shared["trainer"]["world_size"]
        if old_world != self.world and not elastic:
            raise RuntimeError(f"cannot resume {path}: saved with world_size={old_world}, running with {self.world} "
                               "(set training.elastic_resume to reshard)")
        if per_rank and "elastic_rank_states" in per_rank:
            # another world size: optimiser shards are resharded; a rank that existed keeps its RNG streams,
            # a new rank starts from a fresh seed
            states = per_rank["elastic_rank_states"]
            rng = states[self.rank].get("rng") if self.rank < len(states) else None
            if rng is None:
                torch.manual_seed(int(tr.get("seed", 0)) + 104729 * (self.rank + 1) + int(shared["trainer"]["iteration"]))
            self.log.info("elastic resume: world size %d -> %d", old_world, self.world)
        else:
            rng = (per_rank or {}).pop("rng", None) if per_rank else None
        self.model.load_state_dicts(shared, per_rank if per_rank else None)
        if rng is not None:
            torch.set_rng_state(rng["cpu"])
            if rng.get("cuda") is not None and self.device.type == "cuda":
                torch.cuda.set_rng_state(rng["cuda"], self.device)
        for k, s in self.schedules.items():
            s.load_state_dict(shared["trainer"]["schedules"][k])
        self.iteration = int(shared["trainer"]["iteration"])
        self.log.info("resumed from %s (iteration %d)", path, self.iteration)
        return self.iteration

    # ------------------------------------------------------------------ loop
    def train(self):
        self.maybe_resume()
        if self.rank == 0:
            os.makedirs(self.output_dir, exist_ok=True)
            save_config(self.cfg, os.path.join(self.output_dir, "config.yaml"))
        barrier()
        self.log.info("training: iteration %d -> %d, world %d, cp %d", self.iteration, self.max_iters, self.world,
                      self.cp_size)
        for c in self.callbacks:
            c.on_train_start(self, self.iteration)
        self.data = self._build_data(self.cfg.get("data", {}))
        data = iter(self.data)
        prof_cfg = self.cfg.get("profiling")
        with self.timeout, maybe_profile(prof_cfg, self.iteration) as prof, maybe_memory_snapshot(prof_cfg):
            while self.iteration < self.max_iters:
                for c in self.callbacks:
                    c.on_before_dataloading(self, self.iteration)
                batch = next(data)
                for c in self.callbacks:
                    c.on_after_dataloading(self, self.iteration)
                self.last_batch = batch
                out = self.model.training_step(batch, self.iteration)
                phase = self.model.phase_of(self.iteration)
                if phase in self.schedules:
                    self.schedules[phase].step()
                self.iteration += 1
                self.metrics.add(out)
                extra = {}
                for c in self.callbacks:
                    r = c.on_step_end(self, self.iteration, out)
                    if r:
                        extra.update(r)
                self.metrics.add(extra)
                if self.metrics.should_flush(self.iteration) or self.iteration == self.max_iters:
                    rec = self.metrics.flush(self.iteration, {f"lr/{k}": s.get_last_lr()[0]
                                                             for k, s in self.schedules.items()})
                    self.log.info("iter %d/%d %s", self.iteration, self.max_iters,
                                  " ".join(f"{k}={v:.4g}" for k, v in rec.items()
                                           if k.startswith(("dmad", "cm", "dmd", "critic")) and isinstance(v, float)))
                if self.save_every and self.iteration % self.save_every == 0:
                    self.save()
                self.timeout.kick()
                if prof is not None:
                    prof.step()
                if self.dryrun:
                    break
        if self.save_every and self.iteration % self.save_every != 0 and not self.dryrun:
            self.save()
        self.ckpt.finalize()
        for c in self.callbacks:
            c.on_train_end(self, self.iteration)
        if self.device.type == "cuda":
            from ..ops import check_device_status
            check_device_status()
        barrier()
        return self.iteration
