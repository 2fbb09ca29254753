"""The MTP speculative step end to end on the host (CPU).

``LLMEngine`` and ``MTPSpeculator`` run their real host logic (scheduling,
input staging into the workspace buffers, the verify / catch-up / draft body,
acceptance, commit and rollback) on CPU tensors, against a stand-in model:
the target scores the next token of ``x`` with logits 30, 29, 28 at
``7x + 3``, ``7x + 4``, ``7x + 5`` (mod V) and 0 elsewhere, and the drafter
proposes ``7x + 3`` except after multiples of 5. Greedy requests must emit
the argmax chain whatever was accepted; sampling requests must emit one of
the three scored tokens at every step, repeat under the same seed, and leave
the argmax chain.
"""
import types

import torch

from k8v4_xpu_b200.runtime.block_manager import BlockManager
from k8v4_xpu_b200.runtime.scheduler import SamplingParams, Scheduler

V = 997


class _Model:
    def __init__(self):
        self.vocab_start = 0
        self.shape = types.SimpleNamespace(gqa_local=6)

    def forward(self, inp, kv_caches, ws=None, all_rows=False):
        h = inp.input_ids.to(torch.float32).view(-1, 1).repeat(1, 4)
        return h if all_rows else h.index_select(0, inp.logit_rows)

    def logits(self, h):
        x = h[:, 0].to(torch.int64)
        lg = torch.zeros(h.shape[0], V)
        for off, val in ((3, 30.0), (4, 29.0), (5, 28.0)):
            lg.scatter_(1, ((7 * x + off) % V).view(-1, 1), val)
        return lg

    def greedy(self, h):
        return (h[:, 0].to(torch.int64) * 7 + 3) % V

    def mtp_forward(self, hidden, ids, inp, cache, ws=None):
        x = torch.where(ids % 5 == 0, ids + 1, ids)  # the drafter errs after multiples of 5
        return x.to(torch.float32).view(-1, 1).repeat(1, 4)


def _engine(k=6, seqs=2):
    from k8v4_xpu_b200.runtime.engine import LLMEngine
    from k8v4_xpu_b200.runtime.workspace import Workspace
    from k8v4_xpu_b200.spec.mtp import MTPSpeculator
    eng = object.__new__(LLMEngine)  # the engine's host logic without its GPU set-up
    w = k + 1
    eng.cfg = types.SimpleNamespace(cuda_graphs=False, capture_sizes=(), max_num_seqs=seqs, seed=0,
                                    speculative_tokens=k)
    eng.tp = 1
    eng.device = torch.device("cpu")
    eng.blocks = BlockManager(96, block_size=16, page=16, enable_prefix_caching=False)
    eng.scheduler = Scheduler(eng.blocks, max_num_seqs=seqs, max_num_batched_tokens=64, decode_width=w,
                              max_model_len=1024, lookahead=w, mix_prefill_with_decode=False, prefill_slice=32)
    eng.stats = {"steps": 0, "prompt_tokens": 0, "generated_tokens": 0, "prefill_time": 0.0,
                 "decode_time": 0.0, "iteration_tokens": []}
    eng.h2d_bytes = eng.d2h_bytes = 0
    eng.layout = types.SimpleNamespace(hkv=2, gqa=6, page=16)
    eng.max_pages = (1024 + 2 * w + 15) // 16 + 1
    max_tokens = max(64, seqs * w)
    eng.ws = Workspace("cpu", max_tokens, seqs, eng.max_pages, 64, 2, 6, w, 64)
    eng._pin_i64 = torch.zeros(4 * max_tokens, dtype=torch.int64)
    eng._pin_i32 = torch.zeros(2 * (seqs + 1) + seqs * eng.max_pages + max_tokens, dtype=torch.int32)
    eng._pin_out = torch.zeros(max_tokens, dtype=torch.int64)
    eng._h2d_done = None
    eng.kv_caches = [None, None, None]
    eng.graphs = None
    eng.model = _Model()
    eng.mtp = None
    eng.mtp = MTPSpeculator(eng, k, None, seed=0)
    return eng


def _chain(prompt, n):
    out, t = [], prompt[-1]
    for _ in range(n):
        t = (7 * t + 3) % V
        out.append(t)
    return out


def _run(n_tokens=30, seed=7):
    eng = _engine()
    pg, ps = list(range(5, 5 + 45)), list(range(600, 600 + 21))
    g = eng.add_request(pg, SamplingParams(max_tokens=n_tokens, ignore_eos=True))
    s = eng.add_request(ps, SamplingParams(max_tokens=n_tokens, ignore_eos=True, temperature=1.0, seed=seed))
    steps = 0
    while eng.has_unfinished():
        eng.step()
        steps += 1
        assert steps < 200
    eng.blocks.check_invariants()
    return eng, pg, ps, g.output, s.output


def test_mtp_step_on_the_host_greedy_and_sampling():
    eng, pg, ps, g1, s1 = _run()
    assert g1 == _chain(pg, 30)
    prev = ps[-1]
    for t in s1:  # every sampled token is one of the three the target scores
        assert t in {(7 * prev + off) % V for off in (3, 4, 5)}
        prev = t
    # tokens after the first come from the speculative step: some leave the argmax
    off_argmax = sum(1 for a, b in zip(s1, s1[1:]) if b != (7 * a + 3) % V)
    assert off_argmax >= 3
    st = eng.mtp.stats
    assert st.num_drafts > 0 and 0 < st.num_accepted_tokens < st.num_draft_tokens
    _, _, _, g2, s2 = _run()
    assert (g2, s2) == (g1, s1)          # same seeds, same draws
    _, _, _, _, s3 = _run(seed=8)
    assert s3 != s1


def test_plain_engine_step_on_the_host_greedy_and_sampling():
    """The same stand-in without MTP: prefill chunks mixed with decode rows,
    the argmax for greedy requests and seeded draws for sampling ones."""
    def run(seed):
        eng = _engine()
        eng.mtp = None
        eng.scheduler = Scheduler(eng.blocks, max_num_seqs=2, max_num_batched_tokens=24, decode_width=1,
                                  max_model_len=1024)
        pg, ps = list(range(5, 5 + 45)), list(range(600, 600 + 21))
        g = eng.add_request(pg, SamplingParams(max_tokens=20, ignore_eos=True))
        s = eng.add_request(ps, SamplingParams(max_tokens=20, ignore_eos=True, temperature=1.0, seed=seed))
        while eng.has_unfinished():
            eng.step()
        eng.blocks.check_invariants()
        return pg, ps, g.output, s.output

    pg, ps, g1, s1 = run(3)
    assert g1 == _chain(pg, 20)
    prev = ps[-1]
    for t in s1:
        assert t in {(7 * prev + off) % V for off in (3, 4, 5)}
        prev = t
    assert sum(1 for a, b in zip([ps[-1]] + s1, s1) if b != (7 * a + 3) % V) >= 3
    assert run(3)[3] == s1 and run(4)[3] != s1


def _lp_ref(prev, tok):
    x = torch.zeros(V)
    for off, val in ((3, 30.0), (4, 29.0), (5, 28.0)):
        x[(7 * prev + off) % V] = val
    return float(torch.log_softmax(x, -1)[tok])


def test_logprobs_of_every_emitted_token_with_and_without_mtp():
    """A request asking for log-probabilities gets one entry per output
    token: the token's log-probability under the model's logits and the top
    N, from plain steps and from MTP verify rows alike."""
    for mtp in (True, False):
        eng = _engine()
        if not mtp:
            eng.mtp = None
            eng.scheduler = Scheduler(eng.blocks, max_num_seqs=2, max_num_batched_tokens=24, decode_width=1,
                                      max_model_len=1024)
        ps = list(range(600, 600 + 21))
        s = eng.add_request(ps, SamplingParams(max_tokens=17, ignore_eos=True, temperature=1.0, seed=1, logprobs=2))
        g = eng.add_request(list(range(5, 50)), SamplingParams(max_tokens=17, ignore_eos=True))
        while eng.has_unfinished():
            eng.step()
        assert len(s.logprobs) == len(s.output) == 17 and g.logprobs == []
        prev = ps[-1]
        for tok, (lp, top) in zip(s.output, s.logprobs):
            assert abs(lp - _lp_ref(prev, tok)) < 1e-5
            assert [t for t, _ in top] == [(7 * prev + 3) % V, (7 * prev + 4) % V]
            prev = tok
        assert not eng.__dict__.get("_lp_next")  # nothing left waiting


def test_prompt_logprobs_over_chunked_prefill_without_prefix_hits():
    """Prompt log-probabilities: entry k scores prompt token k given the
    ones before it (none for the first), across prefill chunks, with and
    without MTP; such a request takes no prefix-cache hit."""
    for mtp in (True, False):
        eng = _engine()
        eng.blocks = BlockManager(96, block_size=16, page=16, enable_prefix_caching=True)
        if mtp:
            eng.scheduler = Scheduler(eng.blocks, max_num_seqs=2, max_num_batched_tokens=24, decode_width=7,
                                      max_model_len=1024, lookahead=7, mix_prefill_with_decode=False,
                                      prefill_slice=16)
        else:
            eng.mtp = None
            eng.scheduler = Scheduler(eng.blocks, max_num_seqs=2, max_num_batched_tokens=24, decode_width=1,
                                      max_model_len=1024)
        prompt = [int(x) for x in torch.randint(0, V, (53,), generator=torch.Generator().manual_seed(5))]
        first = eng.add_request(prompt, SamplingParams(max_tokens=3, ignore_eos=True))
        while eng.has_unfinished():
            eng.step()
        s = eng.add_request(prompt, SamplingParams(max_tokens=3, ignore_eos=True, prompt_logprobs=2))
        while eng.has_unfinished():
            eng.step()
        assert first.output and s.cached_tokens == 0
        again = eng.add_request(prompt, SamplingParams(max_tokens=3, ignore_eos=True))
        while eng.has_unfinished():
            eng.step()
        assert again.cached_tokens > 0  # the cache holds the prompt: only the logprob request skipped it
        assert len(s.prompt_logprobs) == len(prompt) and s.prompt_logprobs[0] is None
        for k in range(1, len(prompt)):
            lp, top = s.prompt_logprobs[k]
            assert abs(lp - _lp_ref(prompt[k - 1], prompt[k])) < 1e-4
            assert [t for t, _ in top] == [(7 * prompt[k - 1] + 3) % V, (7 * prompt[k - 1] + 4) % V]


def test_repetition_penalty_steers_greedy_tokens_with_and_without_mtp():
    """The stand-in target prefers 7x + 3, then 7x + 4. With the preferred
    token already in the prompt and repetition_penalty 2 (its logit 30 -> 15),
    the greedy choice moves to 7x + 4; plain steps and MTP verify agree."""
    for mtp in (True, False):
        eng = _engine()
        if not mtp:
            eng.mtp = None
            eng.scheduler = Scheduler(eng.blocks, max_num_seqs=2, max_num_batched_tokens=24, decode_width=1,
                                      max_model_len=1024)
        last = 40
        prompt = [(7 * last + 3) % V, 11, last]
        s = eng.add_request(prompt, SamplingParams(max_tokens=6, ignore_eos=True, repetition_penalty=2.0))
        g = eng.add_request(prompt, SamplingParams(max_tokens=6, ignore_eos=True))
        while eng.has_unfinished():
            eng.step()
        assert g.output[0] == (7 * last + 3) % V
        assert s.output[0] == (7 * last + 4) % V
        seen, prev = set(prompt), last
        for tok in s.output:  # every step: the best-scored token not yet seen
            want = next((7 * prev + off) % V for off in (3, 4, 5) if (7 * prev + off) % V not in seen)
            assert tok == want
            seen.add(tok)
            prev = tok


def test_logit_bias_and_min_tokens_with_and_without_mtp():
    for mtp in (True, False):
        eng = _engine()
        if not mtp:
            eng.mtp = None
            eng.scheduler = Scheduler(eng.blocks, max_num_seqs=2, max_num_batched_tokens=24, decode_width=1,
                                      max_model_len=1024)
        last = 40
        forced = eng.add_request([3, last], SamplingParams(max_tokens=5, ignore_eos=True, logit_bias={"77": 100.0}))
        stop = (7 * last + 3) % V  # the target's first choice after the prompt is a stop token here
        held = eng.add_request([3, last], SamplingParams(max_tokens=8, stop_token_ids=(stop,), min_tokens=3))
        free = eng.add_request([3, last], SamplingParams(max_tokens=8, stop_token_ids=(stop,)))
        while eng.has_unfinished():
            eng.step()
        assert forced.output == [77] * 5
        assert free.output == [stop]                      # stops at once
        assert held.output[0] == (7 * last + 4) % V and len(held.output) >= 3


def test_guided_choice_with_and_without_mtp():
    """The output is one of the allowed token sequences, whatever the target
    prefers, and the request stops when a choice is complete."""
    choices = ((11, 12, 13), (11, 14), (20,))
    for mtp in (True, False):
        eng = _engine()
        if not mtp:
            eng.mtp = None
            eng.scheduler = Scheduler(eng.blocks, max_num_seqs=2, max_num_batched_tokens=24, decode_width=1,
                                      max_model_len=1024)
        s = eng.add_request([3, 40], SamplingParams(max_tokens=10, ignore_eos=True, allowed_sequences=choices))
        t = eng.add_request([3, 41], SamplingParams(max_tokens=10, ignore_eos=True, temperature=1.0, seed=2,
                                                    allowed_sequences=choices))
        while eng.has_unfinished():
            eng.step()
        assert tuple(s.output) in choices and tuple(t.output) in choices
        assert s.finish_reason == "stop"
