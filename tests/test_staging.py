"""Decode-step staging into the graph buffers: incremental block-table rows,
table versions, the token view (CPU)."""
import types

import numpy as np
import torch

from k8v4_xpu_b200.runtime.block_manager import BlockManager
from k8v4_xpu_b200.runtime.graphs import prepare_benign, stage_decode_inputs
from k8v4_xpu_b200.runtime.scheduler import SamplingParams, Scheduler, TokenView


def _engine(num_blocks=256, seqs=4, width=64):
    bm = BlockManager(num_blocks, block_size=16)
    sch = Scheduler(bm, max_num_seqs=seqs, max_num_batched_tokens=4096, decode_width=1, lookahead=0,
                    mix_prefill_with_decode=False)
    ws = types.SimpleNamespace(
        input_ids=torch.zeros(64, dtype=torch.int64), positions=torch.zeros(64, dtype=torch.int64),
        slots=torch.zeros(64, dtype=torch.int64), write_en=torch.zeros(seqs, dtype=torch.int64),
        forced_a=torch.zeros(seqs, dtype=torch.int64), cu_q=torch.zeros(seqs + 1, dtype=torch.int32),
        seq_lens=torch.zeros(seqs, dtype=torch.int32), block_table=torch.full((seqs, width), -7, dtype=torch.int32),
        logit_rows=torch.zeros(64, dtype=torch.int64))
    eng = types.SimpleNamespace(ws=ws, blocks=bm, scheduler=sch, _pin_i64=torch.zeros(1024, dtype=torch.int64),
                                _pin_i32=torch.zeros(seqs * width + 64, dtype=torch.int32), device="cpu", h2d_bytes=0)
    return eng


def _prefill(eng, prompt):
    seq = eng.scheduler.add(prompt, SamplingParams(max_tokens=500, ignore_eos=True))
    while True:
        out = eng.scheduler.schedule()
        for c in out.chunks:
            c.seq.computed = c.start + c.num_tokens
            if c.seq.computed >= len(c.seq.prompt) and not c.seq.output:
                c.seq.output.append(1)
        if seq.output:
            return seq


def _decode(eng, n):
    sent = []
    for _ in range(n):
        s = eng.scheduler.schedule()
        before = eng.h2d_bytes
        stage_decode_inputs(eng, s, len(s.chunks), 1)
        sent.append(eng.h2d_bytes - before)
        for c in s.chunks:
            c.seq.computed = c.start + 1
            c.seq.output.append(2)
            eng.blocks.publish(c.seq.seq_id, c.seq.tokens, c.seq.computed)
    return sent


def _row(eng, i, seq):
    """Stage the next step (no commit) and read slot i's device row: a row
    reflects the table as of its staging (a commit may then swap a block for
    an identical published one, which the following staging picks up)."""
    stage_decode_inputs(eng, eng.scheduler.schedule(), 1, 1)
    pages = eng.blocks.page_table(seq.seq_id)
    return eng.ws.block_table[i, :len(pages)].tolist(), pages


def test_rows_extend_incrementally_and_match_the_table():
    eng = _engine()
    a = _prefill(eng, list(range(100)))
    sent = _decode(eng, 40)
    got, want = _row(eng, 0, a)
    assert got == want
    # after the first step only new pages travel: most steps send no table bytes
    small = [b for b in sent[1:] if b <= (3 * 1 + 2) * 8 + 3 * 4 + 4]
    assert len(small) >= len(sent) - 4


def test_truncation_and_new_sequence_rewrite_the_row():
    eng = _engine()
    a = _prefill(eng, list(range(70)))
    _decode(eng, 3)
    v0 = eng.blocks.version[a.seq_id]
    eng.blocks.truncate(a.seq_id, 20)
    assert eng.blocks.version[a.seq_id] > v0
    eng.blocks.ensure(a.seq_id, a.computed + 1)  # fresh blocks after the cut
    _decode(eng, 1)
    got, want = _row(eng, 0, a)
    assert got == want
    # a different sequence in slot 0 gets its own full row
    eng.scheduler.finish(a, "stop")
    eng.blocks.free_seq(a.seq_id)
    b = _prefill(eng, list(range(500, 540)))
    _decode(eng, 2)
    got, want = _row(eng, 0, b)
    assert got == want


def test_prepare_benign_forgets_the_rows():
    eng = _engine()
    a = _prefill(eng, list(range(50)))
    _decode(eng, 2)
    prepare_benign(eng, 1, 1)
    assert eng.ws.block_table[0].abs().sum().item() == 0
    _decode(eng, 1)
    got, want = _row(eng, 0, a)
    assert got == want


def test_token_view():
    v = TokenView([1, 2, 3], [4, 5])
    assert len(v) == 5 and v[-1] == 5 and v[2] == 3 and v[3] == 4
    assert v[1:4] == [2, 3, 4] and v[:2] == [1, 2] and v[3:] == [4, 5] and v[::2] == [1, 3, 5]
    assert list(v) == [1, 2, 3, 4, 5] and v == [1, 2, 3, 4, 5]
    assert np.array_equal(np.asarray(v[0:5]), np.arange(1, 6))


def test_random_serving_keeps_every_staged_row_equal_to_its_table():
    """Sequences come and go (adds with shared prompts, aborts, preemption on
    a small pool, identical blocks swapped in by publish), so batch slots
    change hands; after every staging each slot's device row equals its
    sequence's page table."""
    import random
    for seed in range(8):
        rng = random.Random(seed)
        eng = _engine(num_blocks=rng.choice([10, 16, 40]), seqs=4, width=64)
        sch, bm = eng.scheduler, eng.blocks
        stems = [[rng.randrange(500) for _ in range(rng.randrange(20, 60))] for _ in range(2)]
        for step in range(250):
            if step < 150 and rng.random() < 0.25:
                prompt = list(rng.choice(stems)) + [rng.randrange(500) for _ in range(rng.randrange(0, 20))]
                sch.add(prompt, SamplingParams(max_tokens=rng.randrange(5, 60), ignore_eos=True))
            if step < 150 and sch.running and rng.random() < 0.05:
                sch.abort(rng.choice(list(sch.running)).seq_id)
            s = sch.schedule()
            if not s.chunks:
                continue
            if s.is_decode_only:
                stage_decode_inputs(eng, s, len(s.chunks), 1)
                for i, c in enumerate(s.chunks):
                    pages = bm.page_table(c.seq.seq_id)
                    assert eng.ws.block_table[i, :len(pages)].tolist() == pages, (seed, step, i)
            for c in s.chunks:
                seq = c.seq
                seq.computed = c.start + c.num_tokens
                if c.needs_logits:
                    seq.output.append((seq.tokens[-1] + 1) % 500)
                bm.publish(seq.seq_id, seq.tokens, seq.computed)
                if len(seq.output) >= seq.params.max_tokens:
                    sch.finish(seq, "length")
            bm.check_invariants()
