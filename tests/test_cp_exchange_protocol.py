"""The CP decode partial exchange and the TP GEMM -> all-reduce protocols,
model-checked on the CPU.

Each rank runs, in stream order, for every call c: the attention kernel
(store its partial into its slot of buffer ``c % 2`` on every rank, then add
1 to every rank's counter of that buffer) and the merge (wait until its own
counter holds ``state + world`` signals, read every rank's slot, advance
``state``). The merge's read is split into two steps so that other ranks can
act in between. Random interleavings of the ranks must never let a merge
read a slot that holds another call's partial; with one buffer instead of
two, the check must find such a read (the protocol needs both).
"""
import random

import pytest

from k8v4_xpu_b200.parallel.cp_combine import slot_layout


def _run(world: int, calls: int, buffers: int, seed: int) -> list[str]:
    rng = random.Random(seed)
    data = [[[None] * world for _ in range(buffers)] for _ in range(world)]  # [rank copy][buffer][slot]
    counter = [[0] * buffers for _ in range(world)]
    state = [[0] * buffers for _ in range(world)]
    # per rank: next call and phase (0 store+signal, 1 read begin, 2 read end)
    pc = [[0, 0] for _ in range(world)]
    seen: dict = {}
    errors = []
    while any(c < calls for c, _ in pc):
        ready = []
        for r in range(world):
            c, ph = pc[r]
            if c >= calls:
                continue
            b = slot_layout(c, world, r, 1, 1, buffers)[0]
            if ph == 1 and counter[r][b] < state[r][b] + world:
                continue  # the merge's bounded wait has not been met yet
            ready.append(r)
        assert ready, "deadlock"
        r = rng.choice(ready)
        c, ph = pc[r]
        b = slot_layout(c, world, r, 1, 1, buffers)[0]
        if ph == 0:
            for p in range(world):  # multicast store into every rank's copy, then the signal
                data[p][b][r] = c
            for p in range(world):
                counter[p][b] += 1
            pc[r][1] = 1
        elif ph == 1:
            seen[r] = list(data[r][b])
            pc[r][1] = 2
        else:
            now = list(data[r][b])
            if seen[r] != [c] * world or now != [c] * world:
                errors.append("rank %d call %d read %s then %s" % (r, c, seen[r], now))
            state[r][b] += world
            pc[r] = [c + 1, 0]
    return errors


@pytest.mark.parametrize("world", [2, 4, 8])
def test_two_alternating_buffers_never_expose_another_calls_partial(world):
    for seed in range(200):
        assert _run(world, calls=12, buffers=2, seed=seed) == []


def test_one_buffer_is_not_enough():
    bad = sum(bool(_run(4, calls=12, buffers=1, seed=s)) for s in range(200))
    assert bad > 0


def _run_allreduce(world: int, layers: int, seed: int) -> list[str]:
    """The TP GEMM -> all-reduce protocol: per layer, o_proj adds into slot 0
    of every rank's copy and signals; the norm waits for every rank's signal,
    reads its copy, zeroes it, advances its count; then down_proj does the
    same on slot 1. A rank's adds must never land in a copy that its owner
    has read but not yet zeroed, nor before the owner zeroed the previous use."""
    rng = random.Random(seed)
    copy = [[0, 0] for _ in range(world)]
    counter = [[0, 0] for _ in range(world)]
    state = [[0, 0] for _ in range(world)]
    pc = [[0, 0] for _ in range(world)]  # (op index, phase); op 2l + s = GEMM s of layer l
    seen: dict = {}
    errors = []
    total = 2 * layers
    while any(op < total for op, _ in pc):
        ready = [r for r in range(world) if pc[r][0] < total and not (
            pc[r][1] == 1 and counter[r][pc[r][0] % 2] < state[r][pc[r][0] % 2] + world)]
        assert ready, "deadlock"
        r = rng.choice(ready)
        op, ph = pc[r]
        s = op % 2
        if ph == 0:  # GEMM epilogue: multimem add of this rank's partial (1), then the signal
            for p in range(world):
                copy[p][s] += 1
            for p in range(world):
                counter[p][s] += 1
            pc[r][1] = 1
        elif ph == 1:  # norm: read the sum
            seen[r] = copy[r][s]
            pc[r][1] = 2
        else:  # norm: zero the copy for the next use, advance the count
            if seen[r] != world or copy[r][s] != world:
                errors.append("rank %d op %d read %d, zeroed %d" % (r, op, seen[r], copy[r][s]))
            copy[r][s] = 0
            state[r][s] += world
            pc[r] = [op + 1, 0]
    return errors


@pytest.mark.parametrize("world", [2, 4, 8])
def test_tp_allreduce_slots_never_mix_layers(world):
    for seed in range(200):
        assert _run_allreduce(world, layers=6, seed=seed) == []
