"""Failure detection: store-backed heartbeats and a watchdog.

The reference has no failure detection (switches are scheduled or triggered by a shared-memory flag).  Here
every rank runs a daemon thread that writes ``emb/hb/<rank>`` = wall-clock time into the job's key-value
store every ``interval`` seconds; :class:`Watchdog` reads all heartbeats and reports ranks whose last beat is
older than ``timeout`` (or that never beat).  Detection is entirely on the host: no collective is involved,
so a dead rank cannot make the detector hang.  Recovery is ``ElasticMegatronManager.recover``.

The default store of ``torch.distributed`` is served by rank 0; if rank 0 itself fails, the other ranks'
store calls raise, which :meth:`Watchdog.failed_ranks` reports as ``{0}``.
"""
from __future__ import annotations

import threading
import time
from typing import Iterable, Set

import torch.distributed as dist


def default_store():
    return dist.distributed_c10d._get_default_store()


class Heartbeat:
    def __init__(self, rank: int, store=None, interval: float = 0.2, prefix: str = "emb/hb"):
        self.rank, self.store, self.interval, self.prefix = rank, store or default_store(), interval, prefix
        self._stop = threading.Event()
        self._t = threading.Thread(target=self._run, daemon=True)

    def start(self) -> "Heartbeat":
        self.beat()
        self._t.start()
        return self

    def beat(self) -> None:
        self.store.set(f"{self.prefix}/{self.rank}", repr(time.time()))

    def _run(self):
        while not self._stop.wait(self.interval):
            try:
                self.beat()
            except Exception:  # store gone: stop beating
                return

    def stop(self) -> None:
        self._stop.set()


class Watchdog:
    def __init__(self, ranks: Iterable[int], store=None, timeout: float = 2.0, prefix: str = "emb/hb"):
        self.ranks, self.store, self.timeout, self.prefix = list(ranks), store or default_store(), timeout, prefix

    def failed_ranks(self) -> Set[int]:
        now = time.time()
        dead = set()
        for r in self.ranks:
            try:
                key = f"{self.prefix}/{r}"
                if not self.store.check([key]):
                    dead.add(r)
                    continue
                if now - float(self.store.get(key).decode()) > self.timeout:
                    dead.add(r)
            except Exception:
                dead.add(0 if r != 0 else r)
        return dead

    def wait_for_failure(self, limit: float = 30.0, poll: float = 0.1) -> Set[int]:
        """Poll until some rank is reported failed (bounded by ``limit`` seconds; returns ``set()`` then)."""
        t0 = time.time()
        while time.time() - t0 < limit:
            dead = self.failed_ranks()
            if dead:
                return dead
            time.sleep(poll)
        return set()
