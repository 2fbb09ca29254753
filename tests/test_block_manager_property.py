"""Randomised block-manager runs against a shadow of every block's contents
(CPU). Sequences are allocated (with prefix hits), grow, 'write' their tokens
into their slots, publish, fork (performing the returned copies), roll back
and free. A prefix hit must hand out blocks that hold exactly the tokens it
claims, and no sequence may write into a block that another live sequence or
the cache can still read."""
import random

import pytest

from k8v4_xpu_b200.runtime.block_manager import BlockManager, CapacityError


@pytest.mark.parametrize("seed", range(20))
def test_prefix_hits_serve_the_right_tokens(seed):
    rng = random.Random(seed)
    bs = rng.choice([16, 32])
    bm = BlockManager(rng.choice([6, 12, 40]), block_size=bs)
    content: dict[int, list] = {}          # block -> token written at each offset (None: never)
    seqs: dict[int, dict] = {}             # id -> {"toks": tokens, "done": tokens written}
    stems = [[rng.randrange(50) for _ in range(rng.randrange(bs, 4 * bs))] for _ in range(3)]
    next_id = 0

    def write(sid, upto):
        s = seqs[sid]
        table = bm.tables[sid]
        for pos in range(s["done"], upto):
            b = table[pos // bs]
            # a block being written must be this sequence's alone and unpublished
            assert bm.info[b].ref == 1, ("shared block written", b)
            assert bm.info[b].key is None, ("published block written", b)
            content.setdefault(b, [None] * bs)[pos % bs] = s["toks"][pos]
        s["done"] = upto

    for _ in range(400):
        op = rng.random()
        if op < 0.3:  # a new sequence, often sharing a stem
            toks = list(rng.choice(stems))[:rng.randrange(1, 4 * bs)] + [rng.randrange(50) for _ in range(rng.randrange(0, bs))]
            if not toks:
                continue
            sid = next_id
            next_id += 1
            try:
                cached = bm.allocate(sid, toks)
                bm.ensure(sid, len(toks))
            except CapacityError:
                bm.free_seq(sid)
                continue
            for i, b in enumerate(bm.tables[sid][:cached // bs]):  # hits hold what they claim
                assert content.get(b) == toks[i * bs:(i + 1) * bs], ("stale prefix hit", b)
            seqs[sid] = {"toks": toks, "done": cached}
            write(sid, len(toks))
            bm.publish(sid, toks, len(toks))
        elif op < 0.55 and seqs:  # grow by a few generated tokens
            sid = rng.choice(list(seqs))
            s = seqs[sid]
            new = [rng.randrange(50) for _ in range(rng.randrange(1, bs))]
            try:
                bm.ensure(sid, len(s["toks"]) + len(new))
            except CapacityError:
                continue
            s["toks"] += new
            write(sid, len(s["toks"]))
            bm.publish(sid, s["toks"], len(s["toks"]))
        elif op < 0.65 and seqs:  # fork: share full blocks, copy the tail
            sid = rng.choice(list(seqs))
            s = seqs[sid]
            child = next_id
            next_id += 1
            try:
                copies = bm.fork(sid, child, s["done"])
            except CapacityError:
                continue
            for src, dst in copies:
                content[dst] = list(content.get(src, [None] * bs))
            seqs[child] = {"toks": list(s["toks"]), "done": s["done"]}
        elif op < 0.75 and seqs:  # speculative rollback of unpublished tail tokens
            sid = rng.choice(list(seqs))
            s = seqs[sid]
            keep = max(len(bm.keys[sid]) * bs, s["done"] - rng.randrange(0, bs))
            bm.truncate(sid, keep)
            s["toks"] = s["toks"][:keep]
            s["done"] = keep
        elif seqs:  # finish
            sid = rng.choice(list(seqs))
            bm.free_seq(sid)
            del seqs[sid]
        bm.check_invariants()
