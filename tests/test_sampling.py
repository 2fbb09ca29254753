"""Random sampling (temperature, top-k, top-p, seed) on the host side (CPU)."""
import os
import socket
import traceback
import types

import pytest
import torch
import torch.multiprocessing as mp

from k8v4_xpu_b200.runtime import sampling
from k8v4_xpu_b200.runtime.scheduler import SamplingParams, Sequence


def test_filters_keep_the_top_k_and_the_nucleus():
    x = torch.tensor([3.0, 1.0, 2.0, 0.0, -1.0])
    k2 = sampling.filter_logits(x, 2, 1.0)
    assert torch.isinf(k2[[1, 3, 4]]).all() and torch.equal(k2[[0, 2]], x[[0, 2]])
    p = torch.softmax(x, 0)                        # 0.636, 0.086, 0.234, 0.032, 0.012
    n1 = sampling.filter_logits(x, 0, 0.5)         # the first token alone holds 0.636 >= 0.5
    assert torch.isfinite(n1).tolist() == [True, False, False, False, False]
    n2 = sampling.filter_logits(x, 0, 0.8)         # 0.636 < 0.8: the second-ranked token joins
    assert torch.isfinite(n2).tolist() == [True, False, True, False, False]
    assert float(p[0] + p[2]) >= 0.8
    tiny = sampling.filter_logits(x, 0, 1e-6)      # the most likely token always stays
    assert torch.isfinite(tiny).tolist() == [True, False, False, False, False]
    assert torch.equal(sampling.filter_logits(x, 0, 1.0), x)


def test_greedy_rows_take_the_argmax_and_sampled_rows_follow_the_softmax():
    g = torch.Generator().manual_seed(0)
    logits = torch.randn(3, 50, generator=g)
    greedy = SamplingParams()
    assert sampling.sample_rows(logits, [greedy] * 3, [None] * 3).tolist() == logits.argmax(1).tolist()
    top1 = SamplingParams(temperature=0.7, top_k=1)
    gen = torch.Generator().manual_seed(1)
    assert sampling.sample_rows(logits, [top1] * 3, [gen] * 3).tolist() == logits.argmax(1).tolist()
    # frequencies of 20,000 draws at temperature 0.5 against softmax(logits / 0.5)
    row = torch.tensor([[1.0, 0.5, 0.0, -0.5, -3.0]])
    p = SamplingParams(temperature=0.5)
    gen = torch.Generator().manual_seed(2)
    counts = torch.zeros(5)
    for _ in range(20000):
        counts[sampling.sample_rows(row, [p], [gen])[0]] += 1
    want = torch.softmax(row[0] / 0.5, 0)
    assert (counts / 20000 - want).abs().max() < 0.015


def test_seeds_are_reproducible_and_differ_between_sequences():
    p = SamplingParams(temperature=1.0)
    assert sampling.seed_for(p, 0, 5) == sampling.seed_for(p, 0, 5)
    assert sampling.seed_for(p, 0, 5) != sampling.seed_for(p, 0, 6)
    assert sampling.seed_for(p, 0, 5) != sampling.seed_for(p, 1, 5)
    assert sampling.seed_for(SamplingParams(temperature=1.0, seed=42), 0, 5) == 42
    logits = torch.randn(1, 1000, generator=torch.Generator().manual_seed(3))
    draws = []
    for _ in range(2):
        seq = Sequence(7, [1, 2], SamplingParams(temperature=1.0, seed=123))
        gen = sampling.generator_for(seq, 0, "cpu")
        assert sampling.generator_for(seq, 0, "cpu") is gen  # created once per sequence
        draws.append([int(sampling.sample_rows(logits, [seq.params], [gen])[0]) for _ in range(20)])
    assert draws[0] == draws[1] and len(set(draws[0])) > 1


class _LogitModel:
    """A stand-in whose logits are a fixed function of the hidden row; under
    TP it returns this rank's vocabulary shard."""

    def __init__(self, tp=1, rank=0, vocab=64, comm=None):
        self.tp, self.rank, self.vocab, self.comm = tp, rank, vocab, comm
        self.vocab_start = rank * vocab // tp

    def _full(self, hidden):
        w = torch.arange(self.vocab, dtype=torch.float32)
        return torch.sin(hidden[:, :1] * 0.37 + w * 0.11) * 3.0

    def logits(self, hidden):
        v = self.vocab // self.tp
        return self._full(hidden)[:, self.rank * v:(self.rank + 1) * v]

    def greedy(self, hidden):
        return self._full(hidden).argmax(1)


def _engine(tp=1, rank=0, comm=None, mtp=None):
    from k8v4_xpu_b200.runtime.engine import LLMEngine
    eng = object.__new__(LLMEngine)  # the sampling logic without the GPU set-up
    eng.cfg = types.SimpleNamespace(seed=0)
    eng.tp = tp
    eng.device = torch.device("cpu")
    eng.model = _LogitModel(tp, rank, comm=comm)
    eng.mtp = mtp
    eng.scheduler = types.SimpleNamespace(add=lambda prompt, params: Sequence(0, prompt, params))
    return eng


def test_engine_chooses_argmax_or_seeded_draws_per_row():
    eng = _engine()
    hidden = torch.arange(4, dtype=torch.float32).view(4, 1).repeat(1, 8)
    seqs = [Sequence(i, [1], SamplingParams(temperature=(0.0 if i % 2 == 0 else 1.3), seed=i)) for i in range(4)]
    a = eng._choose(hidden, seqs)
    greedy = eng.model.greedy(hidden)
    assert a[0] == greedy[0] and a[2] == greedy[2]
    seqs2 = [Sequence(i, [1], SamplingParams(temperature=(0.0 if i % 2 == 0 else 1.3), seed=i)) for i in range(4)]
    assert torch.equal(eng._choose(hidden, seqs2), a)      # same seeds, same draws
    assert torch.equal(eng._choose(hidden, None), greedy)  # no sampling request: the argmax kernel path


def test_engine_refuses_bad_params():
    eng = _engine()
    for p in (SamplingParams(temperature=-1.0), SamplingParams(top_p=0.0), SamplingParams(top_k=-2)):
        with pytest.raises(ValueError):
            eng.add_request([1, 2], p)
    eng.add_request([1, 2], SamplingParams(temperature=0.8, top_p=0.9, top_k=40))
    eng.mtp = object()  # sampling requests are served under MTP too (speculative sampling)
    eng.add_request([1, 2], SamplingParams(temperature=0.8))


def test_decode_graphs_leave_sampling_steps_to_the_eager_path():
    from k8v4_xpu_b200.runtime.graphs import DecodeGraphs
    dg = object.__new__(DecodeGraphs)
    dg.width, dg.sizes = 1, [1, 2, 4]

    def sched(*temps):
        return types.SimpleNamespace(chunks=[types.SimpleNamespace(num_tokens=1, seq=Sequence(
            i, [1], SamplingParams(temperature=t))) for i, t in enumerate(temps)])
    assert dg.can_run(sched(0.0, 0.0))
    assert not dg.can_run(sched(0.0, 0.9))


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _tp_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world), LOCAL_RANK=str(rank))
    import torch.distributed as dist
    try:
        from k8v4_xpu_b200.parallel.comm import TPComm, init_from_env
        init_from_env(timeout_s=60, backend="gloo")
        eng = _engine(tp=world, rank=rank, comm=TPComm())
        hidden = torch.arange(6, dtype=torch.float32).view(6, 1).repeat(1, 8)
        seqs = [Sequence(i, [1], SamplingParams(temperature=1.0 if i % 3 else 0.0, top_k=20 if i == 4 else 0))
                for i in range(6)]
        draws = [eng._choose(hidden, seqs).tolist() for _ in range(5)]
        q.put((rank, {"draws": draws, "greedy": eng.model.greedy(hidden).tolist()}))
        dist.barrier()
    except Exception:
        q.put((rank, {"error": traceback.format_exc()}))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


def test_tp_ranks_draw_the_same_tokens_from_gathered_shards():
    """Two gloo ranks, each holding half of the vocabulary: the shards are
    gathered and every rank's generator, seeded alike, draws the same ids."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_tp_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    out = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    for r in range(2):
        assert "error" not in out[r], out[r].get("error")
    assert out[0]["draws"] == out[1]["draws"]
    d = out[0]["draws"]
    for step in d:
        assert [step[i] for i in (0, 3)] == [out[0]["greedy"][i] for i in (0, 3)]  # greedy rows
    assert len({tuple(s) for s in d}) > 1  # the sampled rows vary from step to step
    assert all(0 <= t < 64 for s in d for t in s)


def test_speculative_sampling_keeps_the_target_distribution():
    """With a deterministic drafter, the emitted tokens follow the target's
    sampling distribution: the first token has p_0, and the second, given
    that the first was the draft, has p_1 (Monte Carlo, 40,000 steps)."""
    V, k = 6, 3
    lg = torch.randn(k + 1, V, generator=torch.Generator().manual_seed(0))
    p = SamplingParams(temperature=0.8)
    probs = sampling.probs_rows(lg, p)
    d = torch.tensor([2, 4, 1])
    g = torch.Generator().manual_seed(1)
    N = 40000
    first, second, n2, accepted = torch.zeros(V), torch.zeros(V), 0, 0
    for _ in range(N):
        a, x = sampling.speculative_sample(lg, d, p, g)
        emitted = d[:a].tolist() + [x]
        accepted += a
        first[emitted[0]] += 1
        if len(emitted) > 1 and emitted[0] == int(d[0]):
            second[emitted[1]] += 1
            n2 += 1
    assert (first / N - probs[0]).abs().max() < 0.012
    assert (second / n2 - probs[1]).abs().max() < 0.035
    # the kept fraction of the first draft is p_0(d_0)
    assert abs(n2 / N - float(probs[0, d[0]])) < 0.012 and accepted > 0
    # a draft the target cannot produce (top-k excludes it) is never kept
    pk = SamplingParams(temperature=1.0, top_k=1)
    for _ in range(50):
        a, x = sampling.speculative_sample(lg, torch.tensor([int(lg[0].argmin()), 0, 0]), pk, g)
        assert a == 0 and x == int(lg[0].argmax())


def test_mtp_accept_mixes_greedy_and_sampling_sequences():
    """The verify step's acceptance: greedy sequences keep the draft prefix
    equal to the argmax; sampling ones draw, and t[i, a] holds the drawn token."""
    from k8v4_xpu_b200.spec.mtp import MTPSpeculator
    spec = object.__new__(MTPSpeculator)
    spec.w, spec.k = 4, 3
    eng = _engine()
    spec.eng = eng
    B, w = 2, 4
    hid = torch.arange(B * w, dtype=torch.float32).view(B * w, 1).repeat(1, 8)
    greedy = eng.model.greedy(hid).view(B, w)
    ids = torch.zeros(B, w, dtype=torch.int64)
    ids[0, 1:] = torch.tensor([greedy[0, 0], greedy[0, 1], 7])       # two drafts match the argmax
    ids[1, 1:] = greedy[1, :3]
    seqs = [Sequence(0, [1], SamplingParams()), Sequence(1, [1], SamplingParams(temperature=1.0, seed=5))]
    t, a = spec._accept(hid, ids, B, seqs)
    assert int(a[0]) == 2 and torch.equal(t[0], greedy[0])
    t2, a2 = spec._accept(hid, ids, B, [seqs[0], Sequence(1, [1], SamplingParams(temperature=1.0, seed=5))])
    assert torch.equal(t, t2) and torch.equal(a, a2)  # same seed, same draws
    assert 0 <= int(a[1]) <= 3 and torch.equal(t[1, :int(a[1])], ids[1, 1:1 + int(a[1])])
    tg, ag = spec._accept(hid, ids, B, [Sequence(0, [1], SamplingParams())] * 2)  # no sampling: argmax kernel path
    assert torch.equal(tg, greedy) and int(ag[1]) == 3


def test_penalties_follow_vllm_definitions():
    row = torch.tensor([2.0, -2.0, 1.0, 0.5, -1.0])
    p = SamplingParams(repetition_penalty=2.0)
    got = sampling.process_row(row, [0], [1], p)         # tokens 0 (prompt) and 1 (output) seen
    assert torch.allclose(got, torch.tensor([1.0, -4.0, 1.0, 0.5, -1.0]))
    p = SamplingParams(presence_penalty=0.5, frequency_penalty=0.25)
    got = sampling.process_row(row, [2], [3, 3, 4], p)   # the prompt takes no presence / frequency penalty
    assert torch.allclose(got, torch.tensor([2.0, -2.0, 1.0, 0.5 - 0.5 - 0.5, -1.0 - 0.5 - 0.25]))
    assert not sampling.has_processors(SamplingParams()) and sampling.has_processors(p)
    assert sampling.needs_logits(p)


def test_min_p_logit_bias_and_min_tokens():
    x = torch.tensor([0.0, -0.1, -3.0, -5.0])                 # probabilities ~ .50, .45, .02, .003
    kept = torch.isfinite(sampling.filter_logits(x, 0, 1.0, min_p=0.1)).tolist()
    assert kept == [True, True, False, False]
    row = torch.zeros(6)
    p = SamplingParams(logit_bias={"3": 5.0, "99": 1.0})       # out-of-vocabulary ids are ignored
    assert sampling.process_row(row, [], [], p).tolist() == [0, 0, 0, 5.0, 0, 0]
    p = SamplingParams(min_tokens=2, stop_token_ids=(1, 4))
    assert torch.isinf(sampling.process_row(row, [], [5], p)[[1, 4]]).all()   # one token so far: held back
    assert torch.isfinite(sampling.process_row(row, [], [5, 2], p)).all()     # long enough: free
    assert sampling.has_processors(p) and not sampling.has_processors(SamplingParams(min_p=0.5))
