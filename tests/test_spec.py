"""MTP host logic: forced acceptance, accounting, commit and rollback (CPU)."""
import types

import numpy as np
import pytest

from k8v4_xpu_b200.runtime.block_manager import BlockManager
from k8v4_xpu_b200.runtime.scheduler import SamplingParams, Scheduler
from k8v4_xpu_b200.spec.mtp import MTPSpeculator, SpecStats, forced_accept_prob


def test_forced_accept_prob_solves_mean_length():
    p = forced_accept_prob(3.0, 6)
    assert abs(sum(p ** i for i in range(7)) - 3.0) < 1e-9
    assert forced_accept_prob(7.0, 6) == 1.0
    assert forced_accept_prob(1.0, 6) < 1e-9
    with pytest.raises(ValueError):
        forced_accept_prob(8.0, 6)


def _fake_engine(k=6, forced=3.0, seqs=2, prefill_slice=0):
    cfg = types.SimpleNamespace(cuda_graphs=False, capture_sizes=(), max_num_seqs=seqs)
    bm = BlockManager(64, block_size=16)
    sch = Scheduler(bm, max_num_seqs=seqs, max_num_batched_tokens=256, decode_width=k + 1, lookahead=k + 1,
                    mix_prefill_with_decode=False, prefill_slice=prefill_slice)
    eng = types.SimpleNamespace(cfg=cfg, blocks=bm, scheduler=sch, stats={"generated_tokens": 0})

    def should_stop(seq, tok):
        return len(seq.output) >= seq.params.max_tokens or (
            not seq.params.ignore_eos and tok in seq.params.stop_token_ids)
    eng._should_stop = should_stop
    return eng, MTPSpeculator(eng, k, forced, seed=0)


def test_forced_counts_are_seeded_and_have_the_mean():
    _, a = _fake_engine()
    _, b = _fake_engine()
    ca, cb = a.forced_counts(50000), b.forced_counts(50000)
    assert np.array_equal(ca, cb)
    assert ca.min() >= 0 and ca.max() <= 6
    assert abs(1.0 + ca.mean() - 3.0) < 0.03


def test_commit_emits_accepted_drafts_plus_bonus_and_rolls_back():
    eng, mtp = _fake_engine(forced=None)
    sch = eng.scheduler
    s0 = sch.add(list(range(20)), SamplingParams(max_tokens=50, ignore_eos=True))
    s1 = sch.add(list(range(100, 130)), SamplingParams(max_tokens=3, ignore_eos=True))
    out = sch.schedule()  # prefill both
    for c in out.chunks:
        c.seq.computed = len(c.seq.prompt)
        c.seq.output.append(7)
        c.seq.draft = [1, 2, 3, 4, 5, 6]
    out = sch.schedule()
    assert out.is_decode_only and [c.num_tokens for c in out.chunks] == [7, 7]
    # blocks cover the verify window plus the drafting lookahead
    assert len(eng.blocks.tables[s0.seq_id]) * 16 >= 20 + 14
    t = np.array([[1, 2, 9, 0, 0, 0, 0], [8, 8, 8, 8, 8, 8, 8]])
    acc = np.array([2, 0])
    nd = np.array([[11] * 6, [12] * 6])
    fin = mtp.commit(out, t, acc, nd)
    assert s0.output == [7, 1, 2, 9] and s0.computed == 20 + 3
    assert s0.draft == [11] * 6
    assert s1.output == [7, 8] and s1.computed == 30 + 1
    assert fin == []
    assert mtp.stats.num_drafts == 2 and mtp.stats.num_accepted_tokens == 2
    assert mtp.stats.accepted_per_pos[:3] == [1, 1, 0]
    # s1 hits max_tokens=3 in the middle of an accepted run: the rest is dropped
    out = sch.schedule()
    fin = mtp.commit(out, np.array([[5] * 7, [5] * 7]), np.array([0, 6]), nd)
    assert s1 in fin and len(s1.output) == 3
    eng.blocks.check_invariants()


def test_scheduler_alternates_decode_and_prefill_under_mtp():
    eng, _ = _fake_engine()
    sch = eng.scheduler
    a = sch.add(list(range(20)), SamplingParams(max_tokens=50))
    out = sch.schedule()
    a.computed = 20
    a.output.append(1)
    a.draft = [0] * 6
    sch.add(list(range(40)), SamplingParams(max_tokens=5))
    kinds = []
    for _ in range(4):
        out = sch.schedule()
        kinds.append(out.is_decode_only)
        assert all(c.is_prefill for c in out.chunks) or out.is_decode_only
    assert kinds == [True, False, True, False] or kinds == [False, True, False, True]


def test_scheduler_runs_a_bounded_prefill_slice_beside_mtp_decode():
    eng, _ = _fake_engine(prefill_slice=16)
    sch = eng.scheduler
    a = sch.add(list(range(20)), SamplingParams(max_tokens=50))
    out = sch.schedule()
    assert out.is_decode_only is False and not out.split  # nothing decodes yet: the whole budget prefills
    a.computed = 20
    a.output.append(1)
    a.draft = [0] * 6
    b = sch.add(list(range(40)), SamplingParams(max_tokens=5))
    for want_start in (0, 16, 32):
        out = sch.schedule()
        assert out.split and not out.is_decode_only
        dec, pre = out.parts()
        assert [c.seq for c in dec.chunks] == [a] and dec.is_decode_only and dec.num_tokens == 7
        assert [(c.seq, c.start) for c in pre.chunks] == [(b, want_start)]
        assert pre.num_tokens == min(16, 40 - want_start) and not pre.is_decode_only
        b.computed = want_start + pre.num_tokens
    # b's prompt is done: every step is decode-only again
    b.output.append(3)
    b.draft = [0] * 6
    out = sch.schedule()
    assert out.is_decode_only and not out.split and len(out.chunks) == 2
    with pytest.raises(ValueError):
        Scheduler(eng.blocks, prefill_slice=-1)


def test_spec_stats_mean():
    s = SpecStats(6)
    for a in (0, 6, 2):
        s.record(a)
    assert s.num_draft_tokens == 18 and s.accepted_per_pos == [2, 2, 1, 1, 1, 1]
    assert abs(s.mean_accepted_length - (1 + 8 / 3)) < 1e-12


def test_mtp_catch_up_rows_for_prompt_chunks_and_recompute_prefill():
    from k8v4_xpu_b200.runtime.scheduler import TokenView
    from k8v4_xpu_b200.spec.mtp import next_token_rows
    prompt, output = [10, 11, 12, 13, 14], [20, 21, 22]
    toks = TokenView(prompt, [])
    assert next_token_rows(toks, 0, 3, 5, None) == [11, 12, 13]          # a middle chunk
    assert next_token_rows(toks, 3, 5, 5, 99) == [14, 99]                # last chunk: the sampled token
    # after a preemption the prefill covers prompt + output; the sampled token follows the last output
    toks = TokenView(prompt, output)
    assert next_token_rows(toks, 0, 6, 8, None) == [11, 12, 13, 14, 20, 21]
    assert next_token_rows(toks, 6, 8, 8, 77) == [22, 77]
