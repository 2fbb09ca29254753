"""End-to-end model / engine checks on a tiny random-init decoder (GPU)."""
import pytest
import torch

from k8v4_xpu_b200 import ops
from k8v4_xpu_b200.models.config import TINY
from k8v4_xpu_b200.models.dense import DenseModel, StepInputs
from k8v4_xpu_b200.runtime.engine import EngineConfig, LLMEngine
from k8v4_xpu_b200.runtime.scheduler import SamplingParams

pytestmark = pytest.mark.gpu


def _inputs(prompts, page_of, dev):
    """StepInputs for one prefill of each prompt into scattered pages."""
    ids, pos, slots, cu, lens, rows, tables = [], [], [], [0], [], [], []
    base = 0
    for p in prompts:
        n = len(p)
        npg = (n + 15) // 16
        pages = [page_of(base + i) for i in range(npg)]
        base += npg
        ids += p
        pos += list(range(n))
        slots += [pages[t // 16] * 16 + t % 16 for t in range(n)]
        cu.append(cu[-1] + n)
        lens.append(n)
        rows.append(cu[-1] - 1)
        tables.append(pages)
    W = max(len(t) for t in tables)
    bt = torch.zeros(len(prompts), W, dtype=torch.int32)
    for i, t in enumerate(tables):
        bt[i, :len(t)] = torch.tensor(t)
    return StepInputs(
        input_ids=torch.tensor(ids, device=dev), positions=torch.tensor(pos, device=dev),
        slots=torch.tensor(slots, device=dev), cu_q=torch.tensor(cu, dtype=torch.int32, device=dev),
        seq_lens=torch.tensor(lens, dtype=torch.int32, device=dev), block_table=bt.to(dev),
        logit_rows=torch.tensor(rows, device=dev), max_q_len=max(lens), is_decode=False)


@pytest.mark.parametrize("w4a8", ["w4a16", "w4a8"])
def test_forward_matches_torch_reference(w4a8, monkeypatch):
    monkeypatch.setenv("K8V4_PREFILL_GEMM", w4a8)
    dev = torch.device("cuda")
    m = DenseModel(TINY, device=dev).random_init(seed=3)
    prompts = [list(range(3, 3 + 150)), list(range(100, 100 + 45))]
    inp = _inputs(prompts, lambda i: 2 * i + 1, dev)
    n_pages = 64
    caches = [torch.zeros(n_pages, m.layout.page_bytes, dtype=torch.uint8, device=dev) for _ in m.layers]
    out = m.forward(inp, caches)
    torch.cuda.synchronize()
    assert ops.status() == 0
    ref_caches = [torch.zeros(n_pages, m.layout.page_bytes, dtype=torch.uint8) for _ in m.layers]
    ref = m.reference_forward(inp, ref_caches)
    err = (out.float().cpu() - ref.float()).abs().max().item()
    scale = ref.float().abs().max().item()
    # W4A8 quantizes MLP activations to int8 (the reference path keeps bf16)
    tol = 0.06 if w4a8 == "w4a8" else 0.03
    assert err <= tol * scale, (err, scale)


def test_greedy_logits_match_reference():
    dev = torch.device("cuda")
    m = DenseModel(TINY, device=dev).random_init(seed=4)
    h = torch.randn(3, TINY.hidden, generator=torch.Generator().manual_seed(0)).bfloat16().to(dev)
    lg = m.logits(h).float().cpu()
    from k8v4_xpu_b200.models import gptq
    q, s = gptq.quant_act_rows(h.cpu())
    ref = gptq.w8a8_ref(q, s, m.lm_head.weight.cpu(), m.lm_head.scale.cpu())
    assert (lg - ref).abs().max().item() <= 1e-2 * ref.abs().max().item() + 1e-3
    ids = m.greedy(h)
    assert ids.shape == (3,)


def test_engine_generate_prefill_then_graph_decode():
    cfg = EngineConfig(model="tiny", max_model_len=2048, max_num_seqs=3, max_num_batched_tokens=96,
                       num_kv_blocks=256, device="cuda")
    eng = LLMEngine(cfg, TINY)
    prompts = [list(range(1, 300)), list(range(5, 30)), list(range(9, 170))]
    outs = eng.generate(prompts, SamplingParams(max_tokens=6, ignore_eos=True))
    assert [len(o) for o in outs] == [6, 6, 6]
    assert ops.status() == 0
    assert eng.graphs is not None and eng.graphs.captured
    cfg2 = EngineConfig(model="tiny", max_model_len=2048, max_num_seqs=3, max_num_batched_tokens=96,
                        num_kv_blocks=256, cuda_graphs=False, device="cuda")
    eng2 = LLMEngine(cfg2, TINY)
    outs2 = eng2.generate(prompts, SamplingParams(max_tokens=6, ignore_eos=True))
    assert outs == outs2
    eng.blocks.check_invariants()


def test_prefix_cache_hit_same_tokens():
    cfg = EngineConfig(model="tiny", max_model_len=2048, max_num_seqs=2, max_num_batched_tokens=128,
                       num_kv_blocks=256, device="cuda")
    eng = LLMEngine(cfg, TINY)
    prompt = list(range(11, 11 + 200))
    a = eng.generate([prompt], SamplingParams(max_tokens=5, ignore_eos=True))[0]
    seq = eng.add_request(prompt + [1, 2, 3], SamplingParams(max_tokens=5, ignore_eos=True))
    while eng.has_unfinished():
        eng.step()
    assert seq.cached_tokens >= 192
    b = eng.generate([prompt], SamplingParams(max_tokens=5, ignore_eos=True))[0]
    assert a == b


def test_engine_samples_seeded_rows_beside_greedy_rows():
    """A sampling request (temperature 5, seed) next to a greedy one: the
    sampling steps run eagerly, the seeded draws repeat in a fresh engine,
    they leave the greedy chain, and the greedy request still follows its
    argmax."""
    from test_mtp_gpu import _teacher_forced_margin
    pg, ps = list(range(1, 120)), list(range(7, 90))

    def run():
        cfg = EngineConfig(model="tiny", max_model_len=2048, max_num_seqs=2, max_num_batched_tokens=96,
                           num_kv_blocks=256, device="cuda")
        eng = LLMEngine(cfg, TINY)
        g = eng.add_request(pg, SamplingParams(max_tokens=8, ignore_eos=True))
        s = eng.add_request(ps, SamplingParams(max_tokens=8, ignore_eos=True, temperature=5.0, seed=1234))
        while eng.has_unfinished():
            eng.step()
        assert ops.status() == 0
        return g.output, s.output

    g1, s1 = run()
    g2, s2 = run()
    assert s1 == s2 and len(s1) == 8 and all(0 <= t < TINY.vocab for t in s1)
    m = DenseModel(TINY, device="cuda").random_init(seed=0)
    assert _teacher_forced_margin(m, pg, g1) < 0.05
    assert _teacher_forced_margin(m, ps, s1) > 0.0  # not the argmax chain


def test_engine_reports_logprobs_of_greedy_tokens():
    """A greedy request asking for log-probabilities runs its steps eagerly
    and gets one entry per token: the chosen token holds the top
    log-probability, and the top list is sorted."""
    cfg = EngineConfig(model="tiny", max_model_len=2048, max_num_seqs=2, max_num_batched_tokens=96,
                       num_kv_blocks=256, device="cuda")
    eng = LLMEngine(cfg, TINY)
    s = eng.add_request(list(range(3, 140)), SamplingParams(max_tokens=6, ignore_eos=True, logprobs=3))
    while eng.has_unfinished():
        eng.step()
    assert ops.status() == 0
    assert len(s.logprobs) == len(s.output) == 6
    for tok, (lp, top) in zip(s.output, s.logprobs):
        assert len(top) == 3 and lp <= 0.0
        assert abs(lp - top[0][1]) < 1e-6
        assert top[0][1] >= top[1][1] >= top[2][1]
