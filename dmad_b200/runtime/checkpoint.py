"""Checkpoint / resume with atomic publication, manifests and per-rank optimiser shards.

Parity: the H3 checkpoint index (train/h3/lightx2v_train/runtime/checkpoint.py:5-49:
``checkpoint-<iter>`` directories, completion markers, pruning to ``save_total_limit``, latest
lookup), the DMD trainer's save / resume with world-size and iteration validation
(train/h3/lightx2v_train/trainers/dmd/trainer.py:204-265, base.py:86-98) and the Wan DCP
checkpointer's ``latest_checkpoint.txt`` and optional asynchronous save from pinned host copies
(train/wan/rcm/checkpointers/dcp.py:202-730).

Layout of ``<output_dir>/checkpoint-000000123/``:

    shared.pt          state every rank holds identically (weights, trainer state), written by rank 0
    rank00000.pt ...   state sharded over ranks (fp32 master / moments / EMA shards), one per rank
    config.yaml        the run's config (optional)
    manifest.json      iteration, world size, file sizes, format version
    _SUCCESS           completion marker

A save writes everything into ``checkpoint-<iter>.partial/``; rank 0 writes the manifest and the
marker after every rank has finished, then renames the directory (atomic on one file system) and
updates ``latest_checkpoint.txt``.  A crash mid-save leaves only a ``.partial`` directory, which
lookup ignores and the next save of that iteration replaces.  With ``async_save`` the state is
copied to host memory at the call and written by a background thread; publication happens at the
next ``save`` / ``finalize`` (all ranks), so training continues while the files are written.
"""
from __future__ import annotations

import json
import os
import shutil
import threading
import time

import torch

from ..parallel.dist import barrier, get_rank, get_world_size

FORMAT_VERSION = 1
_PREFIX = "checkpoint-"


def checkpoint_name(iteration: int) -> str:
    return f"{_PREFIX}{iteration:09d}"


def parse_checkpoint_iteration(path: str) -> int:
    return int(os.path.basename(os.path.normpath(path)).split("-")[-1])


def is_complete(path: str) -> bool:
    return os.path.isdir(path) and (os.path.isfile(os.path.join(path, "_SUCCESS"))
                                    or os.path.isfile(os.path.join(path, "trainer_state.pt")))


def completed_checkpoints(output_dir: str) -> list[str]:
    if not os.path.isdir(output_dir):
        return []
    out = []
    for name in os.listdir(output_dir):
        p = os.path.join(output_dir, name)
        if name.startswith(_PREFIX) and not name.endswith(".partial") and is_complete(p):
            try:
                parse_checkpoint_iteration(name)
            except ValueError:
                continue
            out.append(p)
    return sorted(out, key=parse_checkpoint_iteration)


def find_latest_checkpoint(output_dir: str) -> tuple[str | None, int]:
    cks = completed_checkpoints(output_dir)
    if not cks:
        return None, 0
    return cks[-1], parse_checkpoint_iteration(cks[-1])


def prune_checkpoints(output_dir: str, total_limit: int | None):
    """Keep the newest ``total_limit`` completed checkpoints."""
    if total_limit is None or total_limit <= 0:
        return
    cks = completed_checkpoints(output_dir)
    for p in cks[: max(0, len(cks) - total_limit)]:
        shutil.rmtree(p, ignore_errors=True)


def _to_host(obj, pin: bool):
    if torch.is_tensor(obj):
        t = obj.detach()
        if t.is_cuda:
            h = torch.empty(t.shape, dtype=t.dtype, pin_memory=pin)
            h.copy_(t, non_blocking=pin)
            return h
        return t.clone()
    if isinstance(obj, dict):
        return {k: _to_host(v, pin) for k, v in obj.items()}
    if isinstance(obj, (list, tuple)):
        return type(obj)(_to_host(v, pin) for v in obj)
    return obj


def _atomic_save(obj, path: str):
    tmp = path + ".tmp"
    with open(tmp, "wb") as f:
        torch.save(obj, f)
        f.flush()
        os.fsync(f.fileno())
    os.replace(tmp, path)


class CheckpointManager:
    def __init__(self, output_dir: str, total_limit: int | None = None, async_save: bool = False):
        self.output_dir = output_dir
        self.total_limit = total_limit
        self.async_save = async_save
        self._pending: tuple[int, threading.Thread, list] | None = None

    # ------------------------------------------------------------------ save
    def save(self, iteration: int, shared: dict, per_rank: dict | None = None, config_text: str | None = None):
        """Collective: every rank calls with its own ``per_rank`` state (``shared`` is used on rank 0)."""
        self.finalize()
        rank, world = get_rank(), get_world_size()
        final = os.path.join(self.output_dir, checkpoint_name(iteration))
        part = final + ".partial"
        if rank == 0:
            os.makedirs(self.output_dir, exist_ok=True)
            if os.path.exists(part):
                shutil.rmtree(part)
            os.makedirs(part)
        barrier()
        files: list = []

        def write(shared_h, per_rank_h):
            if rank == 0:
                _atomic_save(shared_h, os.path.join(part, "shared.pt"))
                if config_text is not None:
                    with open(os.path.join(part, "config.yaml"), "w") as f:
                        f.write(config_text)
            if per_rank_h is not None:
                _atomic_save(per_rank_h, os.path.join(part, f"rank{rank:05d}.pt"))
            files.append(True)

        pin = torch.cuda.is_available()
        shared_h = _to_host(shared, pin) if rank == 0 else None
        per_rank_h = _to_host(per_rank, pin) if per_rank is not None else None
        if pin:
            torch.cuda.synchronize()
        if self.async_save:
            th = threading.Thread(target=write, args=(shared_h, per_rank_h), daemon=True)
            th.start()
            self._pending = (iteration, th, files, per_rank is not None)
        else:
            write(shared_h, per_rank_h)
            self._publish(iteration, per_rank is not None)

    def finalize(self):
        """Finish and publish a pending asynchronous save (collective)."""
        if self._pending is None:
            return
        iteration, th, files, has_rank = self._pending
        th.join()
        self._pending = None
        if not files:
            raise RuntimeError(f"asynchronous checkpoint write of iteration {iteration} failed")
        self._publish(iteration, has_rank)

    def _publish(self, iteration: int, has_rank_files: bool):
        barrier()
        rank, world = get_rank(), get_world_size()
        final = os.path.join(self.output_dir, checkpoint_name(iteration))
        part = final + ".partial"
        if rank == 0:
            names = sorted(os.listdir(part))
            if has_rank_files:
                missing = [r for r in range(world) if f"rank{r:05d}.pt" not in names]
                if missing:
                    raise RuntimeError(f"checkpoint {iteration}: rank files missing for ranks {missing}")
            manifest = {"iteration": iteration, "world_size": world, "format_version": FORMAT_VERSION,
                        "time": time.time(), "has_rank_files": has_rank_files,
                        "files": {n: os.path.getsize(os.path.join(part, n)) for n in names}}
            with open(os.path.join(part, "manifest.json"), "w") as f:
                json.dump(manifest, f, indent=1)
            open(os.path.join(part, "_SUCCESS"), "w").close()
            if os.path.exists(final):
                shutil.rmtree(final)
            os.replace(part, final)
            with open(os.path.join(self.output_dir, "latest_checkpoint.txt.tmp"), "w") as f:
                f.write(os.path.basename(final))
            os.replace(os.path.join(self.output_dir, "latest_checkpoint.txt.tmp"),
                       os.path.join(self.output_dir, "latest_checkpoint.txt"))
            prune_checkpoints(self.output_dir, self.total_limit)
        barrier()

    # ------------------------------------------------------------------ load
    def latest(self) -> tuple[str | None, int]:
        return find_latest_checkpoint(self.output_dir)

    def load_all_ranks(self, path: str, map_location="cpu") -> list[dict]:
        """Every rank's per-rank state of a checkpoint (elastic resume on another world size)."""
        with open(os.path.join(path, "manifest.json")) as f:
            manifest = json.load(f)
        if not manifest.get("has_rank_files"):
            return []
        return [torch.load(os.path.join(path, f"rank{r:05d}.pt"), map_location=map_location, weights_only=False)
                for r in range(int(manifest["world_size"]))]

    def load(self, path: str, map_location="cpu", elastic: bool = False) -> tuple[dict, dict | None, dict]:
        """(shared, this rank's per-rank state or None, manifest); validates the world size.  With
        ``elastic`` a different world size is accepted and the per-rank state is
        ``{"elastic_rank_states": [every old rank's state]}``."""
        with open(os.path.join(path, "manifest.json")) as f:
            manifest = json.load(f)
        if manifest.get("iteration") != parse_checkpoint_iteration(path):
            raise RuntimeError(f"manifest iteration {manifest.get('iteration')} does not match {path}")
        for name, size in manifest["files"].items():
            p = os.path.join(path, name)
            if not os.path.isfile(p) or os.path.getsize(p) != size:
                raise RuntimeError(f"checkpoint file {p} is missing or truncated")
        shared = torch.load(os.path.join(path, "shared.pt"), map_location=map_location, weights_only=False)
        per_rank = None
        if manifest.get("has_rank_files"):
            world = get_world_size()
            if manifest["world_size"] != world and elastic:
                return shared, {"elastic_rank_states": self.load_all_ranks(path, map_location)}, manifest
            if manifest["world_size"] != world:
                raise RuntimeError(f"checkpoint {path} was saved with world_size={manifest['world_size']}, "
                                   f"resuming with world_size={world} (per-rank optimiser shards; set "
                                   f"training.elastic_resume to reshard them)")
            per_rank = torch.load(os.path.join(path, f"rank{get_rank():05d}.pt"), map_location=map_location,
                                  weights_only=False)
        return shared, per_rank, manifest
