"""Skip layers on the tiny decoder (GPU): layers whose KV stays in fp8 / bf16
pages next to K8/V4 layers, through decode graphs, eager prefill and MTP.

The check is decode-vs-prefill consistency by teacher forcing: one prefill
of prompt + output through the same layers (skip layers included), and each
greedily emitted token must be within a small margin of that position's
maximum logit.
"""
import pytest
import torch

from k8v4_xpu_b200 import ops
from k8v4_xpu_b200.kv import skip_layers as S
from k8v4_xpu_b200.models.config import TINY
from k8v4_xpu_b200.models.dense import StepInputs
from k8v4_xpu_b200.runtime.engine import EngineConfig, LLMEngine
from k8v4_xpu_b200.runtime.scheduler import SamplingParams

pytestmark = pytest.mark.gpu

PROMPTS = [list(range(1, 200)), list(range(5, 30))]


def _engine(**kw):
    base = dict(model="tiny", max_model_len=1024, max_num_seqs=2, max_num_batched_tokens=128,
                num_kv_blocks=128, device="cuda")
    base.update(kw)
    return LLMEngine(EngineConfig(**base), TINY)


def _margin(model, prompt, out):
    """Max over output tokens of (max logit - logit of the emitted token), from
    one prefill with the model's skip layers on plain pages."""
    dev = model.device
    toks = prompt + out[:-1]
    n = len(toks)
    npg = (n + 15) // 16
    cache = [model.skip_kv[i].alloc(npg, dev) if i in model.skip_kv else
             torch.zeros(npg + 1, model.layout.page_bytes, dtype=torch.uint8, device=dev)
             for i in range(len(model.layers))]
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


@pytest.mark.parametrize("name", ["fp8", "bfloat16"])
def test_skip_layer_decode_graphs_agree_with_prefill(name):
    eng = _engine(kv_cache_dtype_skip_layers=(0,), kv_skip_dtype=name)
    lay = S.SkipLayout(eng.model.shape.hkv_local, name)
    assert eng.model.skip_kv == {0: lay}
    assert eng.kv_caches[0].shape[1] == lay.page_bytes
    assert eng.kv_caches[1].shape[1] == eng.layout.page_bytes
    outs = eng.generate(PROMPTS, SamplingParams(max_tokens=16, ignore_eos=True))
    assert ops.status() == 0
    assert [len(o) for o in outs] == [16, 16]
    assert bool(eng.kv_caches[0][:-1].ne(0).any())  # the skip pages were written
    for p, o in zip(PROMPTS, outs):
        assert _margin(eng.model, p, o) < 0.05


def test_mtp_layer_as_a_skip_layer_stays_lossless():
    eng = _engine(speculative_tokens=6, kv_cache_dtype_skip_layers=(TINY.num_layers,), kv_skip_dtype="fp8")
    assert list(eng.model.skip_kv) == [len(eng.model.layers)]
    outs = eng.generate(PROMPTS, SamplingParams(max_tokens=20, ignore_eos=True))
    assert ops.status() == 0
    assert [len(o) for o in outs] == [20, 20]
    for p, o in zip(PROMPTS, outs):
        assert _margin(eng.model, p, o) < 0.05
