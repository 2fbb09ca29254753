"""MTP speculative decoding on the tiny decoder (GPU).

Greedy speculative decoding is lossless: with the verify step accepting only
drafts equal to the target's argmax, every emitted token is the target's
greedy choice given the tokens before it. Token-for-token equality with a
plain engine is too strict a check (a plain engine mixes decode rows into
prefill batches, which run another attention kernel, so near-tied logits can
flip), so losslessness is checked by teacher forcing: one prefill of
prompt + output, and each output token must be within a small margin of
that position's maximum logit.
"""
import pytest
import torch

from k8v4_xpu_b200 import ops
from k8v4_xpu_b200.models.config import TINY
from k8v4_xpu_b200.runtime.engine import EngineConfig, LLMEngine
from k8v4_xpu_b200.runtime.scheduler import SamplingParams

pytestmark = pytest.mark.gpu

PROMPTS = [list(range(1, 300)), list(range(5, 30)), list(range(9, 170))]


def _engine(**kw):
    base = dict(model="tiny", max_model_len=2048, max_num_seqs=3, max_num_batched_tokens=128,
                num_kv_blocks=256, device="cuda")
    base.update(kw)
    return LLMEngine(EngineConfig(**base), TINY)


def _teacher_forced_margin(model, prompt, out):
    """Max over output tokens of (max logit - logit of the emitted token)."""
    from k8v4_xpu_b200.models.dense import StepInputs
    dev = model.device
    toks = prompt + out[:-1]
    n = len(toks)
    npg = (n + 15) // 16
    cache = [torch.zeros(npg + 1, model.layout.page_bytes, dtype=torch.uint8, device=dev)
             for _ in model.layers]
    rows = list(range(len(prompt) - 1, n))
    inp = StepInputs(
        input_ids=torch.tensor(toks, device=dev), positions=torch.arange(n, device=dev),
        slots=torch.arange(n, device=dev), cu_q=torch.tensor([0, n], dtype=torch.int32, device=dev),
        seq_lens=torch.tensor([n], dtype=torch.int32, device=dev),
        block_table=torch.arange(npg, dtype=torch.int32, device=dev).view(1, npg),
        logit_rows=torch.tensor(rows, device=dev), max_q_len=n, is_decode=False)
    lg = model.logits(model.forward(inp, cache)).float()
    picked = lg.gather(1, torch.tensor(out, device=dev).view(-1, 1)).view(-1)
    return (lg.max(1).values - picked).max().item()


def test_mtp_greedy_is_lossless_and_graph_matches_eager():
    params = SamplingParams(max_tokens=24, ignore_eos=True)
    plain = _engine().generate(PROMPTS, params)
    eng = _engine(speculative_tokens=6)
    spec = eng.generate(PROMPTS, params)
    assert ops.status() == 0
    assert [len(o) for o in spec] == [24, 24, 24]
    assert spec[0] == plain[0]
    for p, o in zip(PROMPTS, spec):
        assert _teacher_forced_margin(eng.model, p, o) < 0.05
    assert eng.mtp.graphs, "speculative step did not run as a CUDA graph"
    st = eng.mtp.stats
    assert st.num_drafts > 0 and st.num_draft_tokens == 6 * st.num_drafts
    assert sum(st.accepted_per_pos) == st.num_accepted_tokens
    eager = _engine(speculative_tokens=6, cuda_graphs=False).generate(PROMPTS, params)
    assert eager == spec
    eng.blocks.check_invariants()


def test_mtp_forced_acceptance_mean_length():
    eng = _engine(speculative_tokens=6, forced_accept_mean=3.0, max_num_seqs=4, num_kv_blocks=512)
    prompts = PROMPTS + [list(range(40, 90))]
    outs = eng.generate(prompts, SamplingParams(max_tokens=240, ignore_eos=True))
    assert ops.status() == 0
    assert [len(o) for o in outs] == [240] * 4
    st = eng.mtp.stats
    assert st.num_drafts >= 200
    assert abs(st.mean_accepted_length - 3.0) < 0.35, st.mean_accepted_length
    eng.blocks.check_invariants()


def test_mtp_serves_sampling_requests_by_speculative_sampling():
    """A sampling request (temperature 5, seed) beside a greedy one under
    MTP6: those steps run eagerly with speculative sampling; the seeded
    output repeats in a fresh engine and leaves the argmax chain, and the
    greedy request still follows its argmax."""
    pg, ps = PROMPTS[2], PROMPTS[1]

    def run():
        eng = _engine(speculative_tokens=6)
        g = eng.add_request(pg, SamplingParams(max_tokens=16, ignore_eos=True))
        s = eng.add_request(ps, SamplingParams(max_tokens=16, ignore_eos=True, temperature=5.0, seed=99))
        while eng.has_unfinished():
            eng.step()
        assert ops.status() == 0
        eng.blocks.check_invariants()
        return eng, g.output, s.output

    eng, g1, s1 = run()
    _, g2, s2 = run()
    assert s1 == s2 and len(s1) == 16 and all(0 <= t < TINY.vocab for t in s1)
    assert eng.mtp.stats.num_drafts > 0
    assert _teacher_forced_margin(eng.model, pg, g1) < 0.05
    assert _teacher_forced_margin(eng.model, ps, s1) > 0.0
