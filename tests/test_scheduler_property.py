"""Randomised scheduler + block manager runs (CPU): adds with shared
prefixes (prefix caching), aborts, chunked prefill and preemption on a small
pool. After every step the block invariants hold, every sequence's output
follows the fake model's rule (next = last + 1), no sequence exceeds its
budget, and once adds stop every request drains."""
import random

import pytest

from fakes import FakeEngine
from k8v4_xpu_b200.runtime.scheduler import SamplingParams


preemptions: list[int] = []


@pytest.mark.parametrize("seed", range(12))
def test_random_add_abort_step_keeps_invariants(seed):
    rng = random.Random(seed)
    eng = FakeEngine(max_num_seqs=rng.choice([1, 2, 4]), budget=rng.choice([16, 40, 64]),
                     num_blocks=rng.choice([8, 10, 24]), max_model_len=128)
    prefixes = [[rng.randrange(900) for _ in range(rng.randrange(8, 40))] for _ in range(3)]
    live, done = [], []
    for step in range(200 + 5000):
        if step < 200 and rng.random() < 0.3:
            prompt = list(rng.choice(prefixes)) + [rng.randrange(900) for _ in range(rng.randrange(0, 20))]
            seq = eng.add_request(prompt, SamplingParams(max_tokens=rng.randrange(1, 64), ignore_eos=True))
            live.append(seq)
        if step < 200 and live and rng.random() < 0.05:
            victim = rng.choice(live)
            eng.abort(victim.seq_id)
            live.remove(victim)
        if eng.has_unfinished():
            for seq in eng.step():
                done.append(seq)
                if seq in live:
                    live.remove(seq)
        eng.blocks.check_invariants()
        for seq in live + done:
            assert len(seq.output) <= seq.params.max_tokens
            toks = seq.prompt + seq.output
            for i, t in enumerate(seq.output):  # the fake model's rule
                assert t == (toks[len(seq.prompt) + i - 1] + 1) % eng.vocab, (seq.seq_id, i)
        if step >= 200 and not eng.has_unfinished():
            break
    assert not eng.has_unfinished(), "requests did not drain"
    preemptions.append(eng.scheduler.num_preemptions)
    for seq in done:
        assert len(seq.output) == seq.params.max_tokens


def test_the_random_runs_reached_preemption():
    """The runs above (same module, run first) exercised recompute preemption."""
    if len(preemptions) < 12:
        pytest.skip("run with the parametrised test")
    assert sum(1 for n in preemptions if n > 0) >= 3, preemptions


@pytest.mark.parametrize("prefill_slice", [0, 16])
@pytest.mark.parametrize("seed", range(8))
def test_mtp_shaped_scheduling_keeps_invariants(seed, prefill_slice):
    """The scheduler as MTP6 drives it: decode rows of width 1 + drafts with a
    KV lookahead, decode and prefill steps alternating (``prefill_slice`` 0)
    or decode rows with a bounded prefill slice beside them; a fake verify accepts
    a random number of drafts and emits them plus one token (rollback by
    length, as the real commit does)."""
    from k8v4_xpu_b200.runtime.block_manager import BlockManager
    from k8v4_xpu_b200.runtime.scheduler import Scheduler
    rng = random.Random(seed)
    k, V = 6, 1000
    bm = BlockManager(rng.choice([12, 20, 48]), block_size=16)
    sch = Scheduler(bm, max_num_seqs=4, max_num_batched_tokens=rng.choice([32, 64]), decode_width=k + 1,
                    max_model_len=200, lookahead=k, mix_prefill_with_decode=False, prefill_slice=prefill_slice)
    seqs = []
    for step in range(3000):
        if step < 150 and rng.random() < 0.3:
            prompt = [rng.randrange(V) for _ in range(rng.randrange(1, 60))]
            seqs.append(sch.add(prompt, SamplingParams(max_tokens=rng.randrange(1, 80), ignore_eos=True)))
        if not sch.has_work():
            if step >= 150:
                break
            continue
        out = sch.schedule()
        if out.split:  # decode rows plus prefill chunks: two passes of one step
            dec, pre = out.parts()
            assert dec.chunks and pre.chunks and dec.is_decode_only and not pre.is_decode_only
            assert dec.num_tokens + pre.num_tokens == out.num_tokens
        for c in out.chunks:
            seq = c.seq
            if c.is_prefill:
                seq.computed = c.start + c.num_tokens
                bm.publish(seq.seq_id, seq.tokens, seq.computed)
                if not c.needs_logits:
                    continue
                emitted = [(seq.tokens[-1] + 1) % V]
            else:
                assert c.num_tokens == 1 + len(seq.draft)
                a = rng.randrange(0, len(seq.draft) + 1)
                seq.computed = c.start + a + 1
                emitted = []
                for _ in range(a + 1):
                    emitted.append(((emitted[-1] if emitted else seq.tokens[-1]) + 1) % V)
            for t in emitted:
                seq.output.append(t)
                if len(seq.output) >= seq.params.max_tokens:
                    sch.finish(seq, "length")
                    break
            if not seq.done:
                seq.draft = [rng.randrange(V) for _ in range(k)]
                bm.publish(seq.seq_id, seq.tokens, seq.computed)
        bm.check_invariants()
    assert not sch.has_work()
    for seq in seqs:
        if seq.finish_reason == "abort":
            continue
        assert len(seq.output) == seq.params.max_tokens
        toks = seq.prompt + seq.output
        assert all(toks[len(seq.prompt) + j] == (toks[len(seq.prompt) + j - 1] + 1) % V
                   for j in range(len(seq.output)))
