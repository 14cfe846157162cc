"""Host-side failure detection: iteration timeout and peer heartbeats.

Parity: the Wan trainer's SIGALRM iteration timeout (train/wan/rcm/trainers/trainer_distillation.py:
``signal.alarm(timeout_period)`` re-armed after every successful iteration, with the handler of
train/wan/imaginaire/utils/misc.py:385-388 raising ``TimeoutError``), the ``HeartBeat`` callback
(train/wan/rcm/callbacks/heart_beat.py) and NCCL's heartbeat timeout
(``TORCH_NCCL_HEARTBEAT_TIMEOUT_SEC``, train/wan/imaginaire/utils/distributed.py:64-69).

* ``IterationTimeout`` -- SIGALRM in the main thread; an iteration that runs longer than the
  period raises ``TimeoutError`` there (the process then exits through the normal error path).
* ``Heartbeat`` -- a daemon thread per rank publishes ``time.time()`` under ``hb/<rank>`` in the
  process group's key-value store (or a directory of files) every ``interval`` seconds;
  ``stale_peers(max_age)`` lists ranks whose beat is older than ``max_age`` or missing, and
  ``check(max_age)`` raises ``PeerFailure`` naming them.  A trainer calls ``check`` between steps,
  so a rank that died or hung is detected on the host before the next collective is launched.
  GPU-side waits are bounded separately (device status word).
"""
from __future__ import annotations

import os
import signal
import threading
import time


class PeerFailure(RuntimeError):
    def __init__(self, ranks, ages):
        self.ranks = list(ranks)
        super().__init__(f"no heartbeat from rank(s) {self.ranks} (ages s: {ages})")


class IterationTimeout:
    def __init__(self, period_s: float | None):
        self.period = int(period_s) if period_s else 0
        self._old = None

    def _handler(self, signum, frame):
        raise TimeoutError(f"Timeout error: more than {self.period} seconds passed since the last iteration.")

    def start(self):
        if self.period > 0 and threading.current_thread() is threading.main_thread():
            self._old = signal.signal(signal.SIGALRM, self._handler)
            signal.alarm(self.period)
        return self

    def kick(self):
        """Call after every successful iteration."""
        if self.period > 0 and threading.current_thread() is threading.main_thread():
            signal.alarm(self.period)

    def stop(self):
        if self.period > 0 and threading.current_thread() is threading.main_thread():
            signal.alarm(0)
            if self._old is not None:
                signal.signal(signal.SIGALRM, self._old)

    def __enter__(self):
        return self.start()

    def __exit__(self, *exc):
        self.stop()
        return False


class _FileStore:
    """Minimal key-value store on a shared directory (tests / single-node runs without a group)."""

    def __init__(self, root: str):
        self.root = root
        os.makedirs(root, exist_ok=True)

    def set(self, key: str, value: str):
        p = os.path.join(self.root, key.replace("/", "_"))
        with open(p + ".tmp", "w") as f:
            f.write(value)
        os.replace(p + ".tmp", p)

    def get(self, key: str) -> bytes | None:
        p = os.path.join(self.root, key.replace("/", "_"))
        try:
            with open(p, "rb") as f:
                return f.read()
        except FileNotFoundError:
            return None


class _PGStore:
    def __init__(self, store):
        self.store = store

    def set(self, key, value):
        self.store.set(key, value)

    def get(self, key):
        # check() first: TCPStore.get blocks until the key exists
        if not self.store.check([key]):
            return None
        return self.store.get(key)


def default_store():
    import torch.distributed as dist

    if not (dist.is_available() and dist.is_initialized()):
        return None
    return _PGStore(dist.distributed_c10d._get_default_store())


class Heartbeat:
    def __init__(self, rank: int, world: int, interval_s: float = 5.0, store=None, root: str | None = None,
                 prefix: str = "hb"):
        self.rank, self.world, self.interval = rank, world, float(interval_s)
        self.prefix = prefix
        self.store = store if store is not None else (_FileStore(root) if root else default_store())
        if self.store is None:
            raise ValueError("Heartbeat needs a process group, a store or a directory")
        self._stop = threading.Event()
        self._th = None
        self.t_start = time.time()

    def beat(self):
        self.store.set(f"{self.prefix}/{self.rank}", repr(time.time()))

    def _loop(self):
        while not self._stop.wait(self.interval):
            try:
                self.beat()
            except Exception:  # noqa: BLE001 - the store went away; the peers will notice
                return

    def start(self):
        self.beat()
        self._th = threading.Thread(target=self._loop, name=f"heartbeat-{self.rank}", daemon=True)
        self._th.start()
        return self

    def stop(self):
        self._stop.set()
        if self._th is not None:
            self._th.join(timeout=self.interval + 1)

    def stale_peers(self, max_age_s: float) -> dict[int, float]:
        now = time.time()
        out = {}
        for r in range(self.world):
            if r == self.rank:
                continue
            v = self.store.get(f"{self.prefix}/{r}")
            if v is None:
                age = now - self.t_start  # never seen: count from our own start
            else:
                age = now - float(v.decode() if isinstance(v, bytes) else v)
            if age > max_age_s:
                out[r] = round(age, 2)
        return out

    def check(self, max_age_s: float):
        stale = self.stale_peers(max_age_s)
        if stale:
            raise PeerFailure(stale.keys(), stale)
