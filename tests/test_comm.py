"""TP communicator on CPU (two ``gloo`` ranks as child processes) and the
host side of the context-parallel partial exchange."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world), LOCAL_RANK=str(rank))
    import torch.distributed as dist
    from k8v4_xpu_b200.parallel.comm import TPComm, init_from_env
    import traceback
    try:
        r, w, _ = init_from_env(timeout_s=60, backend="gloo")
        comm = TPComm()
        res = {}
        t = torch.full((4,), float(r + 1))
        res["all_reduce"] = comm.all_reduce(t.clone()).tolist()
        res["all_gather"] = comm.all_gather(torch.tensor([[r, r]], dtype=torch.float32)).tolist()
        res["all_gather_d1"] = comm.all_gather(torch.tensor([[r], [r]], dtype=torch.float32), dim=1).tolist()
        res["reduce_scatter"] = comm.reduce_scatter(torch.arange(4, dtype=torch.float32) * (r + 1)).tolist()
        # row 0: rank 1 wins; row 1: tie -> lowest global index
        val = torch.tensor([1.0, 5.0]) if r == 0 else torch.tensor([2.0, 5.0])
        idx = torch.tensor([10, 30]) if r == 0 else torch.tensor([1010, 7])
        bv, bi = comm.argmax_reduce(val, idx)
        res["argmax"] = (bv.tolist(), bi.tolist())
        res["max_scalar"] = comm.max_scalar(float(r) * 3.5)
        comm.barrier()
        q.put((r, res))
    except Exception:
        q.put((rank, {"error": traceback.format_exc()}))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


def test_tp_comm_gloo_two_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    out = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for r in range(2):
        res = out[r]
        assert "error" not in res, res.get("error")
        assert res["all_reduce"] == [3.0] * 4
        assert res["all_gather"] == [[0.0, 0.0], [1.0, 1.0]]
        assert res["all_gather_d1"] == [[0.0, 1.0], [0.0, 1.0]]
        assert res["argmax"] == ([2.0, 5.0], [1010, 7])
        assert res["max_scalar"] == 3.5
    # sum = [0, 3, 6, 9]; rank r keeps elements 2r, 2r+1
    assert out[0]["reduce_scatter"] == [0.0, 3.0]
    assert out[1]["reduce_scatter"] == [6.0, 9.0]


def test_cp_peer_exchange_slots_and_bounds(monkeypatch):
    """Context-parallel decode exchange through multicast stores: mode switch,
    slot size bound and the two alternating buffers' layout."""
    from k8v4_xpu_b200.parallel import cp_combine as X
    monkeypatch.delenv("K8V4_CP_COMBINE", raising=False)
    assert X.cp_combine_mode() == "peer"
    monkeypatch.setenv("K8V4_CP_COMBINE", "nccl")
    assert X.cp_combine_mode() == "nccl"
    monkeypatch.setenv("K8V4_CP_COMBINE", "ring")
    with pytest.raises(ValueError):
        X.cp_combine_mode()
    # the largest launch the CP engine makes fits: one wave of CTAs, >= 2 splits
    from k8v4_xpu_b200.runtime.engine import decode_splits
    hkv, gqa = 4, 6
    cap = X.max_slot_floats(4, hkv, 1, gqa)
    for B in range(1, 5):
        for pages in (1, 100, 8192, 16384):
            nsplit = max(2, decode_splits(pages, B, hkv))
            assert B * hkv * nsplit * 16 * 130 <= cap
    # buffers alternate; ranks' slots are packed at this call's size
    world, rf, sf = 4, 2080, 10400
    assert X.slot_layout(0, world, 0, rf, sf) == (0, 0, 0)
    assert X.slot_layout(0, world, 3, rf, sf) == (0, 0, 3 * rf)
    assert X.slot_layout(1, world, 2, rf, sf) == (1, world * sf, world * sf + 2 * rf)
    assert X.slot_layout(2, world, 1, rf, sf) == (0, 0, rf)
    # 16-byte aligned multicast addresses (the store kernel's requirement)
    assert all(X.slot_layout(c, world, r, rf, sf)[2] % 4 == 0 for c in range(3) for r in range(world))
    with pytest.raises(ValueError):
        X.slot_layout(0, world, 0, sf + 1, sf)


def test_tp_cp_group_layout():
    from k8v4_xpu_b200.parallel import groups as G
    assert G.tp_members(2, 2) == [[0, 1], [2, 3]] and G.cp_members(2, 2) == [[0, 2], [1, 3]]
    assert G.tp_members(2, 4) == [[0, 1], [2, 3], [4, 5], [6, 7]]
    assert G.cp_members(2, 4) == [[0, 2, 4, 6], [1, 3, 5, 7]]
    assert G.cp_members(1, 8) == [list(range(8))] and G.tp_members(8, 1) == [list(range(8))]
    for tp, cp in ((2, 2), (2, 4), (4, 2)):
        seen = set()
        for r in range(tp * cp):
            t, c = G.coords(r, tp)
            assert r in G.tp_members(tp, cp)[c] and r in G.cp_members(tp, cp)[t]
            assert G.tp_members(tp, cp)[c].index(r) == t and G.cp_members(tp, cp)[t].index(r) == c
            seen.add((t, c))
        assert len(seen) == tp * cp


def _groups_worker(rank, world, port, tp, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world), LOCAL_RANK=str(rank))
    import traceback
    import torch.distributed as dist
    from k8v4_xpu_b200.parallel import groups as G
    from k8v4_xpu_b200.parallel.comm import TPComm, init_from_env
    from k8v4_xpu_b200.parallel.cp import CPGroup
    try:
        r, w, _ = init_from_env(timeout_s=60, backend="gloo")
        pg = G.build(tp, w // tp)
        # the TP communicator and the CP group see their own members only
        tp_sum = TPComm(pg.tp_group).all_reduce(torch.tensor([float(2 ** r)])).item()
        cp = CPGroup(pg.cp_group)
        cp_sum = cp.sum_(torch.tensor([float(2 ** r)])).item()
        q.put((r, {"tp_rank": pg.tp_rank, "cp_rank": pg.cp_rank, "cp_group_rank": cp.rank, "cp_world": cp.world,
                   "tp_sum": tp_sum, "cp_sum": cp_sum}))
    except Exception:
        q.put((rank, {"error": traceback.format_exc()}))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


def test_cp2_by_tp2_groups_on_four_gloo_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_groups_worker, args=(r, 4, port, 2, q)) for r in range(4)]
    for p in procs:
        p.start()
    out = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for r in range(4):
        o = out[r]
        assert "error" not in o, o.get("error")
        t, c = r % 2, r // 2
        assert (o["tp_rank"], o["cp_rank"], o["cp_group_rank"], o["cp_world"]) == (t, c, c, 2)
        assert o["tp_sum"] == sum(2 ** m for m in (2 * c, 2 * c + 1))
        assert o["cp_sum"] == sum(2 ** m for m in (t, t + 2))


def test_cp_page_maps_against_a_brute_force_shard_model():
    """CP block b = C pages: logical page i of a sequence lives on rank i % C
    at physical page blocks[i // C]. Every token's owner, slot, the encoded
    table and each rank's local page list agree with that model."""
    import random
    from k8v4_xpu_b200.parallel.cp import CPGroup, entry
    rng = random.Random(0)
    for _ in range(200):
        C = rng.choice([1, 2, 4, 8])
        n = rng.randrange(1, 400)
        n_pages = (n + 15) // 16
        blocks = rng.sample(range(1000), (n_pages + C - 1) // C)
        groups = []
        for r in range(C):
            g = object.__new__(CPGroup)
            g.rank, g.world = r, C
            groups.append(g)
        for g in groups:
            assert g.encoded_pages(blocks, n) == [entry(i % C, blocks[i // C]) for i in range(n_pages)]
        owned = {r: [] for r in range(C)}
        for p in range(n):
            i = p // 16
            owner = i % C
            for g in groups:
                assert g.owner(p) == owner
                want = blocks[i // C] * 16 + p % 16 if g.rank == owner else -1
                assert g.slot(blocks, p) == want
            owned[owner].append(p)
        for g in groups:
            pages, keys = g.local_pages(blocks, n)
            assert keys == len(owned[g.rank])
            assert pages == [blocks[i // C] for i in range(g.rank, n_pages, C)]
            # local key k of this rank is global token owned[k]: pages in order, 16 per page
            for k, p in enumerate(owned[g.rank]):
                assert pages[k // 16] * 16 + k % 16 == g.slot(blocks, p)


def test_sequence_parallel_tiles_cover_the_chunk_once():
    from k8v4_xpu_b200.parallel.seq_parallel import TILE, owned_rows, tile_owners
    for world in (2, 4, 8):
        for rows in (1, 127, 128, 129, 777, 4224, 4225, 8192):
            t0 = tile_owners(rows, world)
            tiles = -(-rows // TILE)
            assert t0[0] == 0 and t0[-1] == tiles and all(a <= b for a, b in zip(t0, t0[1:]))
            sizes = [b - a for a, b in zip(t0, t0[1:])]
            assert max(sizes) - min(sizes) <= 1  # as even as whole tiles allow
            spans = [owned_rows(rows, t0, o) for o in range(world)]
            assert sum(n for _, n in spans) == rows
            at = 0
            for r0, n in spans:  # contiguous, in rank order
                assert r0 == at or n == 0
                at += n


def test_sequence_parallel_serves_chunks_where_every_rank_owns_a_tile():
    """Smaller chunks (a rank would own no row) take the NCCL all-reduce; the
    engine's fallback depends on `fits` saying so."""
    from k8v4_xpu_b200.parallel.seq_parallel import TILE, SeqParallel, owned_rows, tile_owners
    for world in (2, 4, 8):
        sp = object.__new__(SeqParallel)  # the host bookkeeping only (no buffers)
        sp.world, sp.max_rows, sp.hidden = world, 4224, 5120
        for rows in (1, 96, TILE * world - 1, TILE * world, 4224, 4225):
            ok = sp.fits(rows, 5120)
            assert ok == (TILE * world <= rows <= 4224), (world, rows)
            if ok:
                t0 = tile_owners(rows, world)
                assert all(owned_rows(rows, t0, o)[1] > 0 for o in range(world))
        assert not sp.fits(4224, 4096)


def test_tp_decode_all_reduce_routing(monkeypatch):
    """Which decode calls the fused GEMM -> all-reduce serves: 2-64 rows;
    one-row calls (the decode GEMV) go to NCCL unless K8V4_TP_GEMV_FUSED=1,
    and to the tcgen05 epilogue when the GEMV is switched off."""
    from k8v4_xpu_b200 import ops
    from k8v4_xpu_b200.parallel.fused_ar import FusedAllReduce
    far = object.__new__(FusedAllReduce)  # the routing only (no buffers)
    far.max_rows, far.hidden = 64, 5120
    monkeypatch.delenv("K8V4_TP_GEMV_FUSED", raising=False)
    monkeypatch.delenv("K8V4_DECODE_GEMV", raising=False)
    assert ops.takes_gemv(ops.W4A16, 1, object()) and not ops.takes_gemv(ops.W4A16, 2, object())
    assert not ops.takes_gemv(ops.W4A8, 1, object()) and not ops.takes_gemv(ops.W4A16, 1, None)
    assert not far.fits(1, 5120)
    assert far.fits(2, 5120) and far.fits(64, 5120)
    assert not far.fits(65, 5120) and not far.fits(4, 4096)
    monkeypatch.setenv("K8V4_TP_GEMV_FUSED", "1")
    assert far.fits(1, 5120)
    monkeypatch.delenv("K8V4_TP_GEMV_FUSED")
    monkeypatch.setenv("K8V4_DECODE_GEMV", "0")
    assert not ops.takes_gemv(ops.W4A16, 1, object()) and far.fits(1, 5120)
