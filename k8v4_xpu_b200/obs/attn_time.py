"""Attention device-time accounting without host syncs (opt-in: ``K8V4_ATTN_TIME=1``).

Behaviour of the reference's attention timer (``k8v4_v030/attn_time.py:22-170``):
each decode / prefill attention call is bracketed by CUDA events; a daemon
thread drains events that have completed (``Event.query()``, never a sync)
and keeps per-kind totals, which it publishes to ``K8V4_ATTN_TIME_FILE``
(JSON, one file per rank) every ``interval`` seconds.
"""
from __future__ import annotations

import collections
import contextlib
import json
import os
import threading
import time


class AttnTimer:
    def __init__(self, path: str | None = None, rank: int = 0, interval: float = 1.0, event_factory=None):
        self.path = path or os.environ.get("K8V4_ATTN_TIME_FILE")
        self.rank = rank
        self.interval = interval
        self.pending: collections.deque = collections.deque()
        self.totals = collections.defaultdict(float)   # kind -> ms
        self.counts = collections.defaultdict(int)
        self._lock = threading.Lock()
        self._stop = threading.Event()
        self._thread = None
        if event_factory is None:
            import torch
            event_factory = lambda: torch.cuda.Event(enable_timing=True)  # noqa: E731
        self._event = event_factory

    @contextlib.contextmanager
    def span(self, kind: str):
        a, b = self._event(), self._event()
        a.record()
        try:
            yield
        finally:
            b.record()
            with self._lock:
                self.pending.append((kind, a, b))

    def drain(self) -> int:
        """Fold completed spans into the totals; returns how many were folded."""
        n = 0
        with self._lock:
            while self.pending and self.pending[0][2].query():
                kind, a, b = self.pending.popleft()
                self.totals[kind] += a.elapsed_time(b)
                self.counts[kind] += 1
                n += 1
        return n

    def snapshot(self) -> dict:
        with self._lock:
            return {"rank": self.rank, "total_ms": dict(self.totals), "calls": dict(self.counts),
                    "pending": len(self.pending), "time": time.time()}

    def publish(self) -> None:
        if not self.path:
            return
        p = self.path if "%d" not in self.path else self.path % self.rank
        tmp = p + ".tmp"
        with open(tmp, "w") as f:
            json.dump(self.snapshot(), f)
        os.replace(tmp, p)

    def _run(self) -> None:
        while not self._stop.wait(self.interval):
            self.drain()
            self.publish()

    def start(self) -> "AttnTimer":
        self._thread = threading.Thread(target=self._run, name="k8v4-attn-time", daemon=True)
        self._thread.start()
        return self

    def stop(self) -> None:
        self._stop.set()
        if self._thread is not None:
            self._thread.join(2 * self.interval + 1)
        self.drain()
        self.publish()


TIMER: AttnTimer | None = None


def attention_span(kind: str):
    t = TIMER
    if t is None:
        return contextlib.nullcontext()
    import torch
    if torch.cuda.is_current_stream_capturing():
        return contextlib.nullcontext()
    return t.span(kind)


def install_if_requested(rank: int = 0) -> AttnTimer | None:
    global TIMER
    if os.environ.get("K8V4_ATTN_TIME", "0") not in ("", "0", "false"):
        TIMER = AttnTimer(rank=rank).start()
    return TIMER
