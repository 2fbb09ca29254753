"""The CPU K8/V4 paged decode-attention oracle (CPU)."""

import torch

from k8v4_xpu_b200.kv import layout as L
from k8v4_xpu_b200.kv import oracle as O
from k8v4_xpu_b200.kv.pack import gather_sequence, store_tokens


def test_baseline_oracle_config_matches_bf16_sdpa():
    """4 sequences (1024/2048/3072/4096), 24Q/4KV, D128, page 16, shuffled page
    table, N(0,1) bf16 inputs: one decode step of quantized attention compared
    with unquantized bf16 SDPA."""
    lay = L.b200_layout(4, 6)
    seqs = O.oracle_config(seed=0)
    total_pages = sum((q.shape[0] * 0 + k.shape[0] + 15) // 16 for q, k, v in seqs)
    perm = torch.randperm(total_pages, generator=torch.Generator().manual_seed(0))
    cache = torch.zeros(total_pages, lay.page_bytes, dtype=torch.uint8)
    off = 0
    errs = []
    for q, k, v in seqs:
        n = k.shape[0]
        npg = (n + 15) // 16
        pages = perm[off:off + npg]
        off += npg
        slots = (pages.repeat_interleave(16) * 16 + torch.arange(16).repeat(npg))[:n]
        store_tokens(cache, slots, k, v, lay)
        kd, vd = gather_sequence(cache, pages.tolist(), n, lay)
        out = O.attention_ref(q.float(), kd, vd, [n], lay.gqa)
        ref = O.sdpa_bf16_ref(q, k, v, lay.gqa)
        errs.append((out - ref).abs().max().item())
    # int8 K / int4 V quantization error stays small against unit-variance data
    assert max(errs) < 0.1, errs


def test_list_oracle_matches_tensor_oracle_reference_format():
    """The pure-Python reference-format causal GQA equals the tensor path."""
    q_len, seq = 3, 21
    query = O.deterministic_rows(q_len, 12, seed=1)
    key = O.deterministic_rows(seq, 2, seed=2)
    value = O.deterministic_rows(seq, 2, seed=3)
    out = torch.tensor(O.causal_gqa(query, key, value, seq, q_len))
    lay = L.ref_layout(2)
    kd, vd = O.quant_dequant_kv(torch.tensor(key), torch.tensor(value), lay)
    ends = [L.builtin_q_end(seq, q_len, t) for t in range(q_len)]
    ref = O.attention_ref(torch.tensor(query), kd, vd, ends, 6)
    assert (out - ref).abs().max().item() < 1e-4


def test_empty_query_and_fully_masked_rows():
    assert O.causal_gqa([], [[[0.0] * 256] * 2], [[[0.0] * 256] * 2], 1, 0) == []
    q = torch.randn(2, 6, 128)
    k = torch.randn(4, 1, 128)
    v = torch.randn(4, 1, 128)
    out = O.attention_ref(q, k, v, [0, 2], 6)
    assert torch.equal(out[0], torch.zeros_like(out[0]))
    assert torch.isfinite(out).all()
