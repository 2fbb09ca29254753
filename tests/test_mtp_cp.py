"""MTP under context parallelism: the host side on ``gloo`` ranks (CPU).

The real ``CPEngine`` step logic and ``CPMTPSpeculator`` run on every rank
against a deterministic stand-in model whose target always predicts
``next(tok) = (7 tok + 3) mod V`` and whose drafter is wrong after every
token divisible by 5. The stand-in checks every forward's CP inputs (KV
slots only on the page's owner, per-row visible local key counts) against a
brute-force count. Rank 1's drafter disagrees with rank 0's, as ranks can
when fp32 atomics round differently; the broadcast of rank 0's results must
keep the ranks' outputs identical. Whatever was accepted, the outputs must be
the target's greedy chain, and every rank must take the same collectives (a
mismatch ends in the process group's timeout).
"""
import os
import socket
import traceback
import types

import pytest
import torch
import torch.multiprocessing as mp

V = 997
PROMPTS = [list(range(5, 5 + 83)), list(range(900, 900 + 37))]
MAX_TOKENS = 24


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _target_next(tok: int) -> int:
    return (tok * 7 + 3) % V


def _chain(prompt, n):
    out, t = [], prompt[-1]
    for _ in range(n):
        t = _target_next(t)
        out.append(t)
    return out


class _FakeModel:
    """Hidden row = the row's token (as floats); greedy = the target rule."""

    def __init__(self, eng):
        self.eng = eng
        self.shape = types.SimpleNamespace(gqa_local=6)
        self.vocab_start = 0
        self.checked_rows = 0
        self.prompt_next = {}
        for p in PROMPTS:
            for i in range(len(p) - 1):
                self.prompt_next[p[i]] = p[i + 1]

    def _local(self, n):
        cp = self.eng.cp
        return sum(1 for q in range(n) if (q // 16) % cp.world == cp.rank)

    def _check(self, inp):
        cp = self.eng.cp
        pos = inp.positions.tolist()
        slots = inp.slots.tolist()
        for p, s in zip(pos, slots):
            if s >= 0:
                assert cp.owner(p) == cp.rank and s % 16 == p % 16
            elif inp.is_decode:
                assert cp.owner(p) != cp.rank
        if inp.is_decode:
            cu = inp.cu_q.tolist()
            lens = inp.cp_local_lens.tolist()
            for i in range(len(cu) - 1):
                assert lens[i] == self._local(pos[cu[i + 1] - 1] + 1)
            if inp.q_ends is not None:
                assert inp.q_ends.tolist() == [self._local(p + 1) for p in pos]
            self.checked_rows += len(pos)

    def forward(self, inp, kv_caches, ws, all_rows=False):
        self._check(inp)
        h = inp.input_ids.to(torch.float32).view(-1, 1).repeat(1, 4)
        return h if all_rows else h.index_select(0, inp.logit_rows)

    def greedy(self, h):
        return (h[:, 0].to(torch.int64) * 7 + 3) % V

    def mtp_forward(self, hidden, ids, inp, cache, ws):
        self._check(inp)
        if not inp.is_decode:  # catch-up rows: the token after each prompt position
            for r, (tok, nxt, s) in enumerate(zip(hidden[:, 0].tolist(), ids.tolist(), inp.slots.tolist())):
                if s >= 0 and int(tok) in self.prompt_next:
                    assert nxt == self.prompt_next[int(tok)]
        x = torch.where(ids % 5 == 0, ids + 1, ids)  # wrong after multiples of 5
        if self.eng.cp.rank == 1:
            x = x + 2  # rank 1's drafter disagrees: rank 0's results must win
        return x.to(torch.float32).view(-1, 1).repeat(1, 4)


def _worker(rank, world, port, q, k):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world), LOCAL_RANK=str(rank))
    import torch.distributed as dist
    try:
        from k8v4_xpu_b200.parallel.comm import init_from_env
        from k8v4_xpu_b200.parallel.cp import PAGE, CPGroup
        from k8v4_xpu_b200.runtime.block_manager import BlockManager
        from k8v4_xpu_b200.runtime.cp_engine import CPEngine
        from k8v4_xpu_b200.runtime.scheduler import SamplingParams, Scheduler
        from k8v4_xpu_b200.spec.mtp_cp import CPMTPSpeculator
        init_from_env(timeout_s=60, backend="gloo")
        eng = object.__new__(CPEngine)  # the engine's host logic without its GPU set-up
        eng.cfg = types.SimpleNamespace(cuda_graphs=False, capture_sizes=(), max_num_seqs=2)
        eng.cp = CPGroup()
        eng.device = torch.device("cpu")
        eng.tp = 1
        eng.blocks = BlockManager(64, block_size=PAGE * world, page=PAGE, enable_prefix_caching=False)
        eng.scheduler = Scheduler(eng.blocks, max_num_seqs=2, max_num_batched_tokens=64, decode_width=k + 1,
                                  max_model_len=4096, lookahead=k + 1, mix_prefill_with_decode=False,
                                  prefill_slice=32)
        eng.stats = {"steps": 0, "prompt_tokens": 0, "generated_tokens": 0, "prefill_time": 0.0,
                     "decode_time": 0.0, "iteration_tokens": []}
        eng.h2d_bytes = eng.d2h_bytes = 0
        eng.layout = types.SimpleNamespace(hkv=2, page=PAGE)
        eng.model = _FakeModel(eng)
        eng.kv_caches = [None, None, None]
        eng.ws = None
        eng.cp_graphs = eng.graphs = None
        eng.mtp = CPMTPSpeculator(eng, k, None, seed=0)
        seqs = [eng.add_request(p, SamplingParams(max_tokens=MAX_TOKENS, ignore_eos=True)) for p in PROMPTS]
        steps = 0
        while eng.has_unfinished():
            eng.step()
            steps += 1
            assert steps < 400
        st = eng.mtp.stats
        q.put((rank, {"outs": [s.output for s in seqs], "accepted": st.num_accepted_tokens,
                      "drafts": st.num_drafts, "checked": eng.model.checked_rows, "steps": steps,
                      "h2d": eng.h2d_bytes > 0 and eng.d2h_bytes > 0}))
        dist.barrier()
    except Exception:
        q.put((rank, {"error": traceback.format_exc()}))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_mtp_under_cp_on_gloo_ranks(world):
    k = 6
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q, k)) for r in range(world)]
    for p in procs:
        p.start()
    out = dict(q.get(timeout=180) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    for r in range(world):
        assert "error" not in out[r], out[r].get("error")
        assert out[r]["outs"] == out[0]["outs"]
        assert out[r]["checked"] > 0 and out[r]["h2d"]
        # every rank committed rank 0's accepted counts: same steps, same acceptance
        assert (out[r]["steps"], out[r]["accepted"], out[r]["drafts"]) == \
            (out[0]["steps"], out[0]["accepted"], out[0]["drafts"])
    for p, o in zip(PROMPTS, out[0]["outs"]):
        assert o == _chain(p, MAX_TOKENS)
    # some drafts were accepted, some rejected
    assert 0 < out[0]["accepted"] < out[0]["drafts"] * k


def test_local_keys_and_slots_match_the_page_map():
    from k8v4_xpu_b200.parallel.cp import PAGE, CPGroup, local_keys, local_slots
    for world in (1, 2, 3, 4, 8):
        for rank in range(world):
            g = object.__new__(CPGroup)  # the page-map methods without a process group
            g.rank, g.world = rank, world
            for n in range(0, 400, 7):
                _, keys = g.local_pages(list(range(64)), n)
                assert local_keys(n, rank, world) == keys
            t = torch.arange(0, 400)
            assert local_keys(t, rank, world).tolist() == [local_keys(int(x), rank, world) for x in t]
            blocks = [5, 9, 2, 7]
            blk = torch.tensor([blocks + [0, 0]], dtype=torch.int32).repeat(3, 1)
            nblk = torch.tensor([4, 4, 4])
            for p0 in range(0, PAGE * world * 5, 5):
                pos = torch.tensor([p0, p0 + 1, p0 + 3])
                got = local_slots(blk, nblk, pos, rank, world).tolist()
                for p, s in zip(pos.tolist(), got):
                    if p // (PAGE * world) >= len(blocks):
                        assert s == -1  # past the sequence's blocks
                    else:
                        assert s == g.slot(blocks, p)


def test_verify_rows_merge_to_full_causal_attention():
    """Per-rank partial attention of MTP verify rows, each row seeing the
    first ``local_keys(p + 1)`` keys of the rank's local list, merged over
    the ranks by (m, l, O), equals causal attention over every key (fp32)."""
    from k8v4_xpu_b200.parallel.cp import PAGE, local_keys
    g = torch.Generator().manual_seed(0)
    L, D, w = 16 * 11 + 5, 32, 7
    k = torch.randn(L, D, generator=g)
    v = torch.randn(L, D, generator=g)
    q = torch.randn(w, D, generator=g)
    rows = list(range(L - w, L))  # verify rows at the last w positions
    for world in (2, 3, 4, 8):
        m_all, l_all, o_all = [], [], []
        for r in range(world):
            local = [p for p in range(L) if (p // PAGE) % world == r]  # this rank's keys, page order
            ms, ls, os_ = [], [], []
            for i, p in enumerate(rows):
                n = local_keys(p + 1, r, world)
                vis = local[:n]
                assert vis == [x for x in local if x <= p]  # a prefix of the local list
                if not vis:
                    ms.append(torch.tensor(float("-inf")))
                    ls.append(torch.tensor(0.0))
                    os_.append(torch.zeros(D))
                    continue
                s = k[vis] @ q[i] / D ** 0.5
                m = s.max()
                e = torch.exp(s - m)
                ms.append(m)
                ls.append(e.sum())
                os_.append(e @ v[vis])
            m_all.append(torch.stack(ms))
            l_all.append(torch.stack(ls))
            o_all.append(torch.stack(os_))
        m = torch.stack(m_all)            # [ranks, w]
        M = m.max(0).values
        wgt = torch.exp(m - M)            # exp(-inf) = 0 for a rank with no visible key
        out = (wgt.unsqueeze(-1) * torch.stack(o_all)).sum(0) / (wgt * torch.stack(l_all)).sum(0).unsqueeze(-1)
        for i, p in enumerate(rows):
            s = k[:p + 1] @ q[i] / D ** 0.5
            ref = torch.softmax(s, 0) @ v[:p + 1]
            assert torch.allclose(out[i], ref, atol=1e-5), (world, p)
