"""Context-parallel serving on 2 GPUs: page-sharded KV, peer-page prefill (GPU)."""
import os
import socket
import tempfile
import traceback

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]

PROMPTS = [list(range(5, 5 + 333)), list(range(900, 900 + 70))]


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _log(rank, msg):
    """Progress of a rank, flushed to a file (a stalled rank shows where it
    stopped) in $K8V4_TEST_LOG_DIR, else the system temporary directory."""
    d = os.environ.get("K8V4_TEST_LOG_DIR") or tempfile.gettempdir()
    os.makedirs(d, exist_ok=True)
    with open(os.path.join(d, "k8v4_cp_rank%d.log" % rank), "a") as f:
        f.write(msg + "\n")


def _worker(rank, world, port, q, combine="nccl", graphs=False, spec=0):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank), K8V4_CP_COMBINE=combine, K8V4_CP_GRAPHS="1" if graphs else "0")
    import torch.distributed as dist
    try:
        from k8v4_xpu_b200 import ops
        from k8v4_xpu_b200.models.config import TINY
        from k8v4_xpu_b200.parallel.comm import init_from_env
        from k8v4_xpu_b200.parallel.cp import CPGroup
        from k8v4_xpu_b200.runtime.cp_engine import CPEngine
        from k8v4_xpu_b200.runtime.engine import EngineConfig
        from k8v4_xpu_b200.runtime.scheduler import SamplingParams
        init_from_env(timeout_s=60)
        _log(rank, "init")
        cfg = EngineConfig(model="tiny", context_parallel_size=world, max_model_len=2048, max_num_seqs=2,
                           max_num_batched_tokens=96, num_kv_blocks=96, speculative_tokens=spec,
                           device="cuda:%d" % rank)
        eng = CPEngine(cfg, TINY, CPGroup())
        _log(rank, "engine")
        seqs = [eng.add_request(p, SamplingParams(max_tokens=10, ignore_eos=True)) for p in PROMPTS]
        n = 0
        while eng.has_unfinished():
            eng.step()
            torch.cuda.synchronize()
            n += 1
            _log(rank, "step %d status %d" % (n, ops.status(clear=False)))
        outs = [s.output for s in seqs]
        torch.cuda.synchronize()
        res = {"outs": outs, "status": ops.status(), "peer": eng.cp.peer is not None,
               "graphs": sorted(eng.cp_graphs.graphs) if eng.cp_graphs is not None else None,
               "verify_steps": eng.mtp.stats.num_drafts if eng.mtp is not None else 0}
        if eng.graphs is not None:
            eng.graphs.release()  # graphs holding NCCL calls go before the process group
        q.put((rank, res))
        dist.barrier()
    except Exception:
        _log(rank, traceback.format_exc())
        q.put((rank, {"error": traceback.format_exc()}))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("combine,graphs", [("nccl", False), ("peer", False), ("nccl", True), ("peer", True)])
def test_cp2_generation_matches_tp1_greedy(combine, graphs):
    """Both decode partial exchanges (NCCL all-gather, and multicast stores
    from the attention kernel with a bounded wait in the merge), eager and
    in captured decode graphs."""
    from test_mtp_gpu import _teacher_forced_margin
    from k8v4_xpu_b200.models.config import TINY
    from k8v4_xpu_b200.models.dense import DenseModel
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q, combine, graphs)) for r in range(2)]
    for p in procs:
        p.start()
    out = dict(q.get(timeout=180) for _ in procs)
    for p in procs:
        p.join(timeout=120)
    for r in range(2):
        assert "error" not in out[r], out[r].get("error")
        assert out[r]["status"] == 0
        assert out[r]["peer"] == (combine == "peer")
        if graphs:  # decode steps ran as replays (one graph per batch size seen)
            assert out[r]["graphs"] and set(out[r]["graphs"]) <= {1, 2}
        else:
            assert out[r]["graphs"] is None
    assert out[0]["outs"] == out[1]["outs"]
    m = DenseModel(TINY, device="cuda:0").random_init(seed=0)
    for p, o in zip(PROMPTS, out[0]["outs"]):
        assert len(o) == 10
        assert _teacher_forced_margin(m, p, o) < 0.05


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("combine", ["nccl", "peer"])
def test_cp2_mtp_generation_matches_tp1_greedy(combine):
    """MTP6 under CP2 (spec.mtp_cp): verify rows with per-row local visible
    ends, the MTP layer's pages sharded like the others, drafts from the
    owner's catch-up row. The output is the target's greedy continuation
    whatever the drafter proposes."""
    from test_mtp_gpu import _teacher_forced_margin
    from k8v4_xpu_b200.models.config import TINY
    from k8v4_xpu_b200.models.dense import DenseModel
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q, combine, False, 6)) for r in range(2)]
    for p in procs:
        p.start()
    out = dict(q.get(timeout=240) for _ in procs)
    for p in procs:
        p.join(timeout=120)
    for r in range(2):
        assert "error" not in out[r], out[r].get("error")
        assert out[r]["status"] == 0
        assert out[r]["verify_steps"] > 0
    assert out[0]["outs"] == out[1]["outs"]
    m = DenseModel(TINY, device="cuda:0").random_init(seed=0)
    for p, o in zip(PROMPTS, out[0]["outs"]):
        assert len(o) == 10
        assert _teacher_forced_margin(m, p, o) < 0.05


def _worker_cp_tp(rank, world, port, q, tp):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    import torch.distributed as dist
    try:
        from k8v4_xpu_b200 import ops
        from k8v4_xpu_b200.models.config import TINY
        from k8v4_xpu_b200.parallel import groups
        from k8v4_xpu_b200.parallel.comm import TPComm, init_from_env
        from k8v4_xpu_b200.parallel.cp import CPGroup
        from k8v4_xpu_b200.runtime.cp_engine import CPEngine
        from k8v4_xpu_b200.runtime.engine import EngineConfig
        from k8v4_xpu_b200.runtime.scheduler import SamplingParams
        init_from_env(timeout_s=60)
        pg = groups.build(tp, world // tp)
        cfg = EngineConfig(model="tiny", tensor_parallel_size=tp, context_parallel_size=world // tp,
                           max_model_len=2048, max_num_seqs=2, max_num_batched_tokens=96, num_kv_blocks=96,
                           device="cuda:%d" % rank)
        eng = CPEngine(cfg, TINY, CPGroup(pg.cp_group), rank=pg.tp_rank, comm=TPComm(pg.tp_group))
        _log(rank, "engine cp%d x tp%d" % (world // tp, tp))
        seqs = [eng.add_request(p, SamplingParams(max_tokens=10, ignore_eos=True)) for p in PROMPTS]
        while eng.has_unfinished():
            eng.step()
        torch.cuda.synchronize()
        q.put((rank, {"outs": [s.output for s in seqs], "status": ops.status()}))
        dist.barrier()
    except Exception:
        _log(rank, traceback.format_exc())
        q.put((rank, {"error": traceback.format_exc()}))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 4, reason="needs 4 GPUs")
def test_cp2_by_tp2_generation_matches_tp1_greedy():
    """Context parallelism with tensor parallelism inside each CP rank: the
    TP groups shard the model, the CP groups exchange attention partials."""
    from test_mtp_gpu import _teacher_forced_margin
    from k8v4_xpu_b200.models.config import TINY
    from k8v4_xpu_b200.models.dense import DenseModel
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker_cp_tp, args=(r, 4, port, q, 2)) for r in range(4)]
    for p in procs:
        p.start()
    out = dict(q.get(timeout=240) for _ in procs)
    for p in procs:
        p.join(timeout=120)
    for r in range(4):
        assert "error" not in out[r], out[r].get("error")
        assert out[r]["status"] == 0
        assert out[r]["outs"] == out[0]["outs"]
    m = DenseModel(TINY, device="cuda:0").random_init(seed=0)
    for p, o in zip(PROMPTS, out[0]["outs"]):
        assert len(o) == 10
        assert _teacher_forced_margin(m, p, o) < 0.05
