"""The engine thread behind the HTTP server, and the TP follower loop.

One thread owns the engine (nothing else touches it): it drains submitted
commands (add / abort), runs ``engine.step()`` while there is work, and pushes
each request's new tokens to that request's asyncio queue. Under tensor or
context parallelism every rank runs the same engine; rank 0 broadcasts the
step's commands over a CPU (gloo) group before applying them, so every rank
schedules identically and issues the same collectives in the same order. The
broadcast also runs while idle (every ``idle_s``), which doubles as a
heartbeat: a follower whose rank 0 died ends with the group's timeout
instead of waiting forever. (In the reference this is vLLM's own engine
loop and TP workers, ``k8v4_v030/launch.sh:176-194``.)
"""
from __future__ import annotations

import dataclasses
import queue
import threading
import time
import traceback

from ..runtime.scheduler import SamplingParams


@dataclasses.dataclass
class RequestHandle:
    rid: int
    prompt: list[int]
    params: SamplingParams
    loop: object = None          # asyncio loop of the HTTP handler
    out: object = None           # asyncio.Queue of (new_ids, finished, reason, new_logprobs or None)
    seq: object = None
    emitted: int = 0
    arrival: float = dataclasses.field(default_factory=time.monotonic)


class TPControl:
    """Broadcasts rank 0's step commands to the follower ranks (gloo group)."""

    def __init__(self, group=None):
        import torch.distributed as dist
        self.dist = dist
        self.group = group
        self.rank = dist.get_rank()

    def exchange(self, cmds):
        obj = [cmds if self.rank == 0 else None]
        self.dist.broadcast_object_list(obj, src=0, group=self.group)
        return obj[0]


def apply_commands(engine, cmds, seqs: dict, handles: dict | None = None, on_reject=None) -> None:
    """Apply one step's commands in order. ``seqs`` maps request id -> sequence
    on every rank (followers add requests in the same order, so ids agree).
    A request the engine refuses (``ValueError``: empty, too long) is
    dropped on every rank alike and reported through ``on_reject``; it does
    not stop the engine."""
    for c in cmds:
        if c[0] == "add":
            _, rid, prompt, params = c
            try:
                seq = engine.add_request(prompt, SamplingParams(**params))
            except ValueError as e:
                if on_reject is not None:
                    on_reject(rid, str(e))
                continue
            seqs[rid] = seq
            if handles is not None and rid in handles:
                handles[rid].seq = seq
        elif c[0] == "abort":
            seq = seqs.pop(c[1], None)
            if seq is not None and not seq.done:
                engine.abort(seq.seq_id)


class EngineDriver:
    def __init__(self, engine, metrics=None, control: TPControl | None = None, idle_s: float = 0.05,
                 status_every: int = 16, watchdog=None):
        self.engine = engine
        self.watchdog = watchdog
        self.metrics = metrics
        self.control = control
        self.idle_s = idle_s
        self.status_every = status_every
        self._cmds: queue.Queue = queue.Queue()
        self._handles: dict[int, RequestHandle] = {}
        self._seqs: dict = {}
        self._next = 0
        self._lock = threading.Lock()
        self._stop = threading.Event()
        self._thread = threading.Thread(target=self._run, name="k8v4-engine", daemon=True)
        self.error: str | None = None
        self.steps = 0

    @property
    def healthy(self) -> bool:
        return self.error is None and self._thread.is_alive()

    def start(self) -> "EngineDriver":
        self._thread.start()
        return self

    def stop(self, timeout: float = 10.0) -> None:
        self._stop.set()
        self._thread.join(timeout)

    def submit(self, prompt: list[int], params: SamplingParams, loop=None, out=None) -> RequestHandle:
        if self.error is not None:
            raise RuntimeError("engine failed: %s" % self.error.splitlines()[-1])
        with self._lock:
            rid = self._next
            self._next += 1
        h = RequestHandle(rid, list(prompt), params, loop, out)
        self._handles[rid] = h
        self._cmds.put(("add", rid, list(prompt), dataclasses.asdict(params)))
        return h

    def abort(self, h: RequestHandle) -> None:
        self._cmds.put(("abort", h.rid))

    # ------------------------------------------------------------ engine side
    def _drain(self, block: bool) -> list:
        cmds = []
        try:
            cmds.append(self._cmds.get(timeout=self.idle_s) if block else self._cmds.get_nowait())
            while True:
                cmds.append(self._cmds.get_nowait())
        except queue.Empty:
            pass
        return cmds

    def _emit(self, h: RequestHandle, new: list[int], finished: bool, reason: str | None, lps=None) -> None:
        if h.out is None:
            return
        item = (new, finished, reason, lps)
        if h.loop is not None:
            h.loop.call_soon_threadsafe(h.out.put_nowait, item)
        else:
            h.out.put_nowait(item)

    def _publish(self, finished_seqs) -> None:
        done_ids = {s.seq_id for s in finished_seqs}
        for rid, h in list(self._handles.items()):
            seq = h.seq
            if seq is None:
                continue
            new = seq.output[h.emitted:]
            fin = seq.seq_id in done_ids or seq.done
            if new or fin:
                lps = list(seq.logprobs[h.emitted:len(seq.output)]) if seq.params.logprobs is not None else None
                h.emitted = len(seq.output)
                self._emit(h, list(new), fin, seq.finish_reason if fin else None, lps)
            if fin:
                if self.metrics is not None:
                    self.metrics.observe_finished(seq)
                del self._handles[rid]
                self._seqs.pop(rid, None)

    def _reject(self, rid: int, msg: str) -> None:
        h = self._handles.pop(rid, None)
        if h is not None:
            self._emit(h, [], True, "rejected: " + msg)

    def _fail_all(self, msg: str) -> None:
        for rid, h in list(self._handles.items()):
            self._emit(h, [], True, "error")
            del self._handles[rid]

    def _run(self) -> None:
        eng = self.engine
        try:
            while not self._stop.is_set():
                idle = not eng.has_unfinished()
                cmds = self._drain(block=idle)
                if self.control is not None:
                    cmds = self.control.exchange(cmds + ([("stop",)] if self._stop.is_set() else []))
                apply_commands(eng, cmds, self._seqs, self._handles, on_reject=self._reject)
                if self.watchdog is not None:
                    self.watchdog.guard()  # a lost rank stops us before the next launch
                if eng.has_unfinished():
                    finished = eng.step()
                    self.steps += 1
                    if self.status_every and self.steps % self.status_every == 0:
                        check_device_status()
                    self._publish(finished)
                    if self.metrics is not None:
                        self.metrics.observe_engine(eng)
                else:
                    self._publish([])
            if self.control is not None:
                self.control.exchange([("stop",)])
        except Exception:
            self.error = traceback.format_exc()
            self._fail_all(self.error)


def check_device_status() -> None:
    """Raise when a kernel recorded an error (a bounded wait that gave up, a
    rejected shape): the step's results cannot be trusted."""
    from .. import ops
    if not ops.available():
        return
    st = ops.status()
    if st:
        raise DeviceStatusError(st)


class DeviceStatusError(RuntimeError):
    def __init__(self, status: int):
        code, site = status & 0xFF, status >> 8
        names = {1: "mbarrier wait timed out", 2: "peer wait timed out", 3: "bad shape", 4: "bad index"}
        super().__init__("device status 0x%x: %s (site %d)" % (status, names.get(code, "error"), site))
        self.status = status


def follower_loop(engine, control: TPControl, watchdog=None) -> None:
    """Ranks > 0: mirror rank 0's commands and steps until it says stop."""
    seqs: dict = {}
    while True:
        cmds = control.exchange(None)
        if any(c[0] == "stop" for c in cmds):
            return
        apply_commands(engine, cmds, seqs)
        if watchdog is not None:
            watchdog.guard()
        for rid in [r for r, q in seqs.items() if q.done]:
            del seqs[rid]
        if engine.has_unfinished():
            engine.step()
