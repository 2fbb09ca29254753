"""Tensor parallel forward and serving on 2, 4 and 8 GPUs (NCCL), checked
against TP1.

Each rank is a child process with its own GPU. Every rank draws the full
random-init matrices from one seed and keeps its shard, so the TPn model is
the TP1 model split by heads / MLP columns / vocab rows. The test model has
the 27B head structure (24 query / 4 KV heads of 128): at TP8 each KV head is
replicated on two ranks and the per-rank GQA is 3.

    torchrun is not needed: ``python -m pytest tests/test_tp_gpu.py -m gpu``
    spawns the ranks itself (one per GPU, rendezvous on 127.0.0.1).
"""
import os
import socket
import traceback

import pytest
import torch
import torch.multiprocessing as mp

from k8v4_xpu_b200.models.config import ModelConfig

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _prefill_inputs(prompts, dev):
    from k8v4_xpu_b200.models.dense import StepInputs
    ids, pos, slots, cu, lens, rows, tables = [], [], [], [0], [], [], []
    base = 0
    for p in prompts:
        n = len(p)
        npg = (n + 15) // 16
        pages = [base + i for i in range(npg)]
        base += npg
        ids += p
        pos += list(range(n))
        slots += [pages[t // 16] * 16 + t % 16 for t in range(n)]
        cu.append(cu[-1] + n)
        lens.append(n)
        rows.append(cu[-1] - 1)
        tables.append(pages)
    W = max(len(t) for t in tables)
    bt = torch.zeros(len(prompts), W, dtype=torch.int32)
    for i, t in enumerate(tables):
        bt[i, :len(t)] = torch.tensor(t)
    return StepInputs(
        input_ids=torch.tensor(ids, device=dev), positions=torch.tensor(pos, device=dev),
        slots=torch.tensor(slots, device=dev), cu_q=torch.tensor(cu, dtype=torch.int32, device=dev),
        seq_lens=torch.tensor(lens, dtype=torch.int32, device=dev), block_table=bt.to(dev),
        logit_rows=torch.tensor(rows, device=dev), max_q_len=max(lens), is_decode=False)


PROMPTS = [list(range(3, 3 + 150)), list(range(100, 100 + 45))]
# the 27B head structure at test size: TP 2/4/8 all divide it, TP8 replicates KV heads
TP_MODEL = ModelConfig(name="tp-test", num_layers=2, hidden=1024, num_heads=24, num_kv_heads=4, head_dim=128,
                       intermediate=2048, vocab=8192, max_position=8192)
SMALL_PROMPTS = [list(range(3, 3 + 40)), list(range(100, 100 + 17))]
def _sp_prompts(world):
    """Two prompts whose chunk gives every rank at least one 128-row tile and
    a ragged last tile."""
    n = 128 * world + 37
    return [list(range(3, 3 + n // 2)), list(range(100, 100 + n - n // 2))]


TINY_PROMPTS = [[5]]  # one row: the decode GEMV and its multicast all-reduce epilogue


def _log(rank, msg):
    """Progress of a rank, flushed to a file (a stalled rank shows where it
    stopped) in $K8V4_TEST_LOG_DIR, else the system temporary directory."""
    import tempfile
    d = os.environ.get("K8V4_TEST_LOG_DIR") or tempfile.gettempdir()
    os.makedirs(d, exist_ok=True)
    with open(os.path.join(d, "k8v4_tp_rank%d.log" % rank), "a") as f:
        f.write(msg + "\n")


def _collect(procs, q, timeout_s=420):
    """Results of every rank; fails (instead of waiting out the timeout) as
    soon as a rank process has died without reporting."""
    import queue
    import time
    out = {}
    t0 = time.monotonic()
    while len(out) < len(procs):
        try:
            r, res = q.get(timeout=5)
            out[r] = res
            continue
        except queue.Empty:
            pass
        dead = [i for i, p in enumerate(procs) if i not in out and p.exitcode is not None]
        if dead:
            raise AssertionError("rank(s) %s exited (codes %s) without a result" %
                                 (dead, [procs[i].exitcode for i in dead]))
        if time.monotonic() - t0 > timeout_s:
            raise AssertionError("ranks %s gave no result in %d s" %
                                 (sorted(set(range(len(procs))) - set(out)), timeout_s))
    return out


def _worker(rank, world, port, q):
    import faulthandler
    import tempfile
    d = os.environ.get("K8V4_TEST_LOG_DIR") or tempfile.gettempdir()
    os.makedirs(d, exist_ok=True)
    # a crash of the rank (signal) leaves its Python stack in the rank's log
    fault_log = open(os.path.join(d, "k8v4_tp_rank%d.log" % rank), "a")
    faulthandler.enable(file=fault_log, all_threads=True)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank), NCCL_NVLS_ENABLE="0",
                      # the opt-in paths are covered too: the one-row multicast GEMV
                      # epilogue and the sequence-parallel prefill
                      K8V4_TP_GEMV_FUSED="1", K8V4_TP_PREFILL="sp")
    import torch.distributed as dist
    try:
        from k8v4_xpu_b200 import ops
        from k8v4_xpu_b200.models.dense import DenseModel
        from k8v4_xpu_b200.parallel.comm import TPComm, init_from_env
        from k8v4_xpu_b200.runtime.engine import EngineConfig, LLMEngine
        from k8v4_xpu_b200.runtime.scheduler import SamplingParams
        init_from_env(timeout_s=120)
        comm = TPComm()
        dev = torch.device("cuda", rank)
        torch.cuda.set_device(dev)
        _log(rank, "tp%d start" % world)
        m = DenseModel(TP_MODEL, tp=world, rank=rank, device=dev, comm=comm).random_init(seed=3)
        inp = _prefill_inputs(PROMPTS, dev)
        caches = [torch.zeros(64, m.layout.page_bytes, dtype=torch.uint8, device=dev) for _ in m.layers]
        hid = m.forward(inp, caches)
        ids = m.greedy(hid)
        res = {"hidden": hid.float().cpu(), "ids": ids.cpu(), "logits": m.logits(hid).float().cpu()}
        _log(rank, "prefill (nccl all-reduce) done")
        # prefill with the residual sharded by token rows between the fused
        # GEMM -> reduce-scatter and all-gather -> GEMM kernels (twice: the
        # running signal counts must keep matching), on a chunk where every
        # rank owns at least one 128-row tile (smaller ones take NCCL)
        from k8v4_xpu_b200.parallel.seq_parallel import SeqParallel
        sp_prompts = _sp_prompts(world)
        sp_inp = _prefill_inputs(sp_prompts, dev)
        sp_pages = sum((len(p_) + 15) // 16 for p_ in sp_prompts)
        caches = [torch.zeros(sp_pages, m.layout.page_bytes, dtype=torch.uint8, device=dev) for _ in m.layers]
        res["hidden_sp_ref"] = m.forward(sp_inp, caches).float().cpu()
        m.sp = SeqParallel(None, dev, sum(len(p_) for p_ in sp_prompts), TP_MODEL.hidden)
        for _ in range(2):
            caches = [torch.zeros(sp_pages, m.layout.page_bytes, dtype=torch.uint8, device=dev) for _ in m.layers]
            res["hidden_sp"] = m.forward(sp_inp, caches).float().cpu()
        res["sp_calls"] = m.sp.calls
        _log(rank, "sequence-parallel prefill done")
        m.sp = None
        # decode-sized batch (<= 64 rows): the GEMM -> all-reduce runs fused (NVLS multicast adds)
        from k8v4_xpu_b200.parallel.fused_ar import FusedAllReduce
        small = _prefill_inputs(SMALL_PROMPTS, dev)
        caches = [torch.zeros(64, m.layout.page_bytes, dtype=torch.uint8, device=dev) for _ in m.layers]
        res["small_nccl"] = m.forward(small, caches).float().cpu()
        _log(rank, "small rows (nccl) done")
        m.fused_ar = FusedAllReduce(None, dev, 64, TP_MODEL.hidden)
        for _ in range(3):  # repeated uses: the running signal counts must keep matching
            caches = [torch.zeros(64, m.layout.page_bytes, dtype=torch.uint8, device=dev) for _ in m.layers]
            res["small_fused"] = m.forward(small, caches).float().cpu()
        # a single row: the row-parallel GEMMs run as the decode GEMV with its
        # multicast all-reduce epilogue
        _log(rank, "small rows (fused all-reduce) done")
        tiny = _prefill_inputs(TINY_PROMPTS, dev)
        caches = [torch.zeros(64, m.layout.page_bytes, dtype=torch.uint8, device=dev) for _ in m.layers]
        res["tiny_fused"] = m.forward(tiny, caches).float().cpu()
        m.fused_ar, far = None, m.fused_ar
        caches = [torch.zeros(64, m.layout.page_bytes, dtype=torch.uint8, device=dev) for _ in m.layers]
        res["tiny_nccl"] = m.forward(tiny, caches).float().cpu()
        m.fused_ar = far
        torch.cuda.synchronize(dev)
        _log(rank, "one row (GEMV all-reduce and nccl) done")
        res["fused_calls"] = m.fused_ar.calls
        res["kv_heads"] = m.shape.kv_heads_of(rank, TP_MODEL.num_kv_heads)
        res["gqa_local"] = m.shape.gqa_local
        cfg = EngineConfig(model="tp-test", tensor_parallel_size=world, max_model_len=2048, max_num_seqs=2,
                           max_num_batched_tokens=96, num_kv_blocks=128, device=str(dev))
        eng = LLMEngine(cfg, TP_MODEL, comm=comm, rank=rank)
        _log(rank, "engine built")
        res["gen"] = eng.generate(PROMPTS, SamplingParams(max_tokens=8, ignore_eos=True))
        _log(rank, "generate done")
        res["graph"] = bool(eng.graphs and eng.graphs.captured)
        res["comm_mode"] = eng.tp_comm_mode
        res["prefill_mode"] = eng.tp_prefill_mode
        res["status"] = ops.status()
        eng.graphs.release()
        comm.barrier()
        q.put((rank, res))
    except Exception:
        _log(rank, traceback.format_exc())
        q.put((rank, {"error": traceback.format_exc()}))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4, 8])
def test_tp_matches_tp1(world):
    if torch.cuda.device_count() < world:
        pytest.skip("needs %d GPUs" % world)
    from k8v4_xpu_b200.models.dense import DenseModel
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    try:
        out = _collect(procs, q)
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.exitcode is None:
                p.kill()
    for r in range(world):
        assert "error" not in out[r], out[r].get("error")
        assert out[r]["status"] == 0 and out[r]["graph"]
    # KV heads: split while TP divides them, then each one shared by TP / 4 ranks (GQA 3)
    rep = max(1, world // TP_MODEL.num_kv_heads)
    for r in range(world):
        assert out[r]["kv_heads"] == ([r // rep] if rep > 1 else list(range(r * 4 // world, (r + 1) * 4 // world)))
        assert out[r]["gqa_local"] == (3 if world == 8 else 6)
    # ranks agree exactly (replicated residual stream, reduced argmax)
    for r in range(1, world):
        assert torch.equal(out[0]["hidden"], out[r]["hidden"]), r
        assert torch.equal(out[0]["small_fused"], out[r]["small_fused"]), r
        assert out[0]["gen"] == out[r]["gen"], r
    assert out[0]["fused_calls"] == 4 * 2 * TP_MODEL.num_layers
    for r in range(1, world):
        assert torch.equal(out[0]["tiny_fused"], out[r]["tiny_fused"]), r
    # the fused path adds the ranks' fp32 partials; the NCCL path rounds each
    # rank's partial row and the sum to bf16 (two layers, one row)
    ref_tiny = out[0]["tiny_nccl"]
    err = (out[0]["tiny_fused"] - ref_tiny).abs().max().item()
    assert err <= 0.05 * ref_tiny.abs().max().item(), err
    assert out[0]["comm_mode"] == "fused" and out[0]["prefill_mode"] == "sp"
    # sequence-parallel prefill: 4 fused GEMMs per layer, ranks agree exactly,
    # and it matches the NCCL all-reduce path up to bf16 partial sums
    assert out[0]["sp_calls"] == 2 * 4 * TP_MODEL.num_layers
    for r in range(1, world):
        assert torch.equal(out[0]["hidden_sp"], out[r]["hidden_sp"]), r
    # (each rank's partial rows reach the owner as bf16 and are summed there;
    # the NCCL path rounds the GEMM output and the all-reduced sum instead)
    err = (out[0]["hidden_sp"] - out[0]["hidden_sp_ref"]).abs().max().item()
    assert err <= 0.03 * out[0]["hidden_sp_ref"].abs().max().item(), err
    ref_small = out[0]["small_nccl"]
    err = (out[0]["small_fused"] - ref_small).abs().max().item()
    assert err <= 0.02 * ref_small.abs().max().item(), err
    # TPn vs TP1 on the same weights: reduction order differs, values agree closely
    dev = torch.device("cuda", 0)
    m = DenseModel(TP_MODEL, device=dev).random_init(seed=3)
    inp = _prefill_inputs(PROMPTS, dev)
    caches = [torch.zeros(64, m.layout.page_bytes, dtype=torch.uint8, device=dev) for _ in m.layers]
    ref = m.forward(inp, caches).float().cpu()
    err = (out[0]["hidden"] - ref).abs().max().item()
    assert err <= 0.03 * ref.abs().max().item(), err
    lg_ref = m.logits(m.forward(inp, caches)).float().cpu()
    full = torch.cat([out[r]["logits"] for r in range(world)], 1)  # the vocab shards side by side
    assert full.shape == lg_ref.shape
    assert (full - lg_ref).abs().max().item() <= 0.03 * lg_ref.abs().max().item()
    picked = lg_ref.gather(1, out[0]["ids"].view(-1, 1)).view(-1)
    assert ((lg_ref.max(1).values - picked) < 0.05).all()
