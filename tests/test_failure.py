"""Failure detection without GPU faults: failures made on the host, gloo ranks (CPU)."""
import os
import socket
import time
import traceback

import torch
import torch.multiprocessing as mp

from k8v4_xpu_b200.api.driver import DeviceStatusError
from k8v4_xpu_b200.parallel.health import CommTimeout, Heartbeat, Watchdog


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _send(q, rank, msg):
    """Put and flush before the process exits (os._exit skips the queue's feeder thread)."""
    q.put((rank, msg))
    q.close()
    q.join_thread()


def _init(rank, world, port, timeout_s):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    from k8v4_xpu_b200.parallel.comm import init_from_env
    init_from_env(timeout_s=timeout_s, backend="gloo")


def _peer_exits(rank, world, port, q):
    import torch.distributed as dist
    try:
        _init(rank, world, port, 4)
        if rank == 1:
            _send(q, rank, "exited")
            os._exit(0)  # leaves without joining the collective
        t0 = time.monotonic()
        try:
            dist.all_reduce(torch.ones(4))
            _send(q, rank, "no error")
        except Exception as e:
            _send(q, rank, "error after %.1f s: %s" % (time.monotonic() - t0, type(e).__name__))
    except Exception:
        _send(q, rank, traceback.format_exc())
    os._exit(0)


def _silent_rank(rank, world, port, q):
    import torch.distributed as dist
    try:
        _init(rank, world, port, 60)
        store = dist.distributed_c10d._get_default_store()
        hb = Heartbeat(store, rank, world, interval=0.1).start()
        wd = Watchdog(hb, timeout=1.0)
        dist.barrier()
        if rank == 1:
            hb.stop()   # still alive, no longer beating (a hung rank)
            time.sleep(6)
            _send(q, rank, "done")
            os._exit(0)
        wd.guard()      # both alive at first
        t0 = time.monotonic()
        while time.monotonic() - t0 < 5:
            try:
                wd.guard()
            except CommTimeout as e:
                _send(q, rank, "timeout %s after %.1f s" % (e.ranks, time.monotonic() - t0))
                os._exit(0)
            time.sleep(0.1)
        _send(q, rank, "not detected")
    except Exception:
        _send(q, rank, traceback.format_exc())
    os._exit(0)


def _dropped_broadcast(rank, world, port, q):
    import torch.distributed as dist
    from k8v4_xpu_b200.api.driver import TPControl
    try:
        _init(rank, world, port, 60)
        ctl = TPControl(dist.new_group(backend="gloo", timeout=__import__("datetime").timedelta(seconds=3)))
        if rank == 0:
            time.sleep(8)  # rank 0 drops the step's command message
            _send(q, rank, "done")
            os._exit(0)
        t0 = time.monotonic()
        try:
            ctl.exchange(None)
            _send(q, rank, "received")
        except Exception as e:
            _send(q, rank, "error after %.1f s: %s" % (time.monotonic() - t0, type(e).__name__))
    except Exception:
        _send(q, rank, traceback.format_exc())
    os._exit(0)


def _run(fn, world=2, wait=60):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=fn, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = {}
    deadline = time.monotonic() + wait
    while len(out) < world and time.monotonic() < deadline:
        try:
            r, msg = q.get(timeout=1)
            out[r] = msg
        except Exception:
            pass
    for p in procs:
        p.join(timeout=15)
        if p.is_alive():
            p.kill()
    return out


def test_collective_errors_when_a_peer_exits():
    out = _run(_peer_exits)
    assert out.get(1) == "exited"
    assert out.get(0, "").startswith("error after"), out
    assert float(out[0].split()[2]) < 30


def test_watchdog_names_the_silent_rank():
    out = _run(_silent_rank)
    assert out.get(0, "").startswith("timeout [1]"), out


def test_dropped_command_broadcast_times_out():
    out = _run(_dropped_broadcast)
    assert out.get(1, "").startswith("error after"), out


def test_device_status_decoding():
    e = DeviceStatusError(2 | (201 << 8))
    assert "peer wait timed out" in str(e) and "site 201" in str(e)
    e = DeviceStatusError(1 | (207 << 8))
    assert "mbarrier" in str(e)
