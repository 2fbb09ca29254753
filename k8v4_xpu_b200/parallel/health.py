"""Failure detection between ranks: heartbeats, a watchdog, and timeouts.

Three layers, none of which needs a GPU fault to be exercised:

* device: every spin-wait in the kernels is bounded (``K8V4_WAIT_LIMIT_NS``);
  a wait that gives up records an error code and site in the library's status
  word and the kernel returns. The host reads it (``ops.status()``) and the
  engine driver raises :class:`~k8v4_xpu_b200.api.driver.DeviceStatusError`;
* collectives: process groups are created with short timeouts, so a collective
  whose peer died or never joins ends with an error instead of waiting
  forever;
* host: each rank's :class:`Heartbeat` thread bumps a counter in the
  rendezvous store; :class:`Watchdog` checks the others' counters before each
  step and raises :class:`CommTimeout` naming the ranks that stopped, so the
  survivors learn of a lost rank before their next launch.

The reference has a launcher health wait with a deadline and container-exit
detection (``k8v4_v030/launch.sh:219-232``) and nothing between ranks; these
layers are what a one-process-per-GPU job needs in its place.
"""
from __future__ import annotations

import threading
import time


class CommTimeout(RuntimeError):
    def __init__(self, msg: str, ranks: list[int] | None = None):
        super().__init__(msg)
        self.ranks = ranks or []


class Heartbeat:
    """Publishes ``<prefix>/<rank>`` = a counter and a wall-clock stamp every ``interval`` s."""

    def __init__(self, store, rank: int, world: int, interval: float = 0.5, prefix: str = "k8v4/hb"):
        self.store, self.rank, self.world = store, rank, world
        self.interval, self.prefix = interval, prefix
        self.count = 0
        self._stop = threading.Event()
        self._thread = threading.Thread(target=self._run, name="k8v4-heartbeat", daemon=True)

    def key(self, r: int) -> str:
        return "%s/%d" % (self.prefix, r)

    def beat(self) -> None:
        self.count += 1
        self.store.set(self.key(self.rank), "%d:%.6f" % (self.count, time.time()))

    def _run(self) -> None:
        while not self._stop.is_set():
            try:
                self.beat()
            except Exception:
                return
            self._stop.wait(self.interval)

    def start(self) -> "Heartbeat":
        self.beat()
        self._thread.start()
        return self

    def stop(self) -> None:
        self._stop.set()
        self._thread.join(2 * self.interval + 1)


class Watchdog:
    """Raises :class:`CommTimeout` when another rank's heartbeat is older than ``timeout`` s."""

    def __init__(self, heartbeat: Heartbeat, timeout: float = 5.0):
        self.hb = heartbeat
        self.timeout = timeout
        self._seen: dict[int, tuple[int, float]] = {}  # rank -> (count, local time it changed)
        self._t0 = time.monotonic()

    def stale_ranks(self) -> list[int]:
        now = time.monotonic()
        stale = []
        for r in range(self.hb.world):
            if r == self.hb.rank:
                continue
            count = -1
            if self.hb.store.check([self.hb.key(r)]):
                raw = self.hb.store.get(self.hb.key(r)).decode()
                count = int(raw.split(":", 1)[0])
            prev = self._seen.get(r)
            if prev is None or count != prev[0]:
                self._seen[r] = (count, now)
                changed = now
            else:
                changed = prev[1]
            since = now - (changed if count >= 0 else self._t0)
            if since > self.timeout:
                stale.append(r)
        return stale

    def guard(self) -> None:
        stale = self.stale_ranks()
        if stale:
            raise CommTimeout("no heartbeat from rank(s) %s for %.1f s" % (stale, self.timeout), stale)
