"""Batch planner, backend guards and the eager paged-prefill oracle (CPU)."""
import math

import pytest
import torch

from k8v4_xpu_b200.attention import plan
from k8v4_xpu_b200.attention.backend import K8V4AttentionBackend, K8V4AttentionImpl, K8V4MetadataBuilder
from k8v4_xpu_b200.attention.reference import SDPA_MAX_KEYS, attention_dense, eager_prefill, paged_prefill
from k8v4_xpu_b200.kv import oracle as O
from k8v4_xpu_b200.kv.layout import b200_layout
from k8v4_xpu_b200.kv.pack import gather_sequence, store_tokens


def test_uniform_packed_decode_classification():
    assert plan.uniform_packed_q_len([1, 1, 1]) == 1
    assert plan.uniform_packed_q_len([7, 7]) == 7
    assert plan.uniform_packed_q_len([7, 1]) is None
    assert plan.uniform_packed_q_len([11]) == 10 + 0 or plan.uniform_packed_q_len([11]) is None
    assert plan.uniform_packed_q_len([10], gqa=6) == 10
    assert plan.uniform_packed_q_len([11], gqa=6) is None  # 66 rows > 64
    assert plan.uniform_packed_q_len([21], gqa=3) == 21
    assert plan.uniform_packed_q_len([]) is None
    assert plan.query_segments([0, 3, 3, 10]) == [(0, 3), (3, 3), (3, 10)]
    with pytest.raises(ValueError):
        plan.query_segments([1, 2])
    with pytest.raises(ValueError):
        plan.query_segments([0, 5, 4])
    assert plan.decode_workspace_floats(4, 4, 37, 1, 6) == 4 * 4 * 37 * 16 * 130


def test_decoder_contract_guards():
    lay = plan.require_decoder(128, 24, 4)
    assert (lay.hkv, lay.gqa) == (4, 6)
    for kw in ({"sliding_window": 4096}, {"alibi_slopes": [1.0]}, {"logits_soft_cap": 30.0},
               {"attn_type": "encoder"}, {"sinks": torch.zeros(4)}):
        with pytest.raises(NotImplementedError):
            plan.require_decoder(128, 24, 4, **kw)
    with pytest.raises(NotImplementedError):
        plan.require_decoder(256, 24, 4)
    with pytest.raises(ValueError):
        plan.require_decoder(128, 24, 5)


def test_backend_shape_and_metadata():
    B = K8V4AttentionBackend
    assert B.get_kv_cache_shape(10, 32, 4, 128) == (20, 4 * 3232)
    assert B.state_bytes_per_token(4) == 808
    with pytest.raises(ValueError):
        B.get_kv_cache_shape(10, 32, 4, 128, "fp8")
    bld = K8V4MetadataBuilder(24, 4, device="cpu")
    md = bld.build([1, 1], [100, 2000], [list(range(7)), list(range(125))], [99, 1999])
    assert md.is_decode and md.num_decode_tokens == 2 and md.nsplit == min(148 // 8, 16)
    md = bld.build([30, 1], [30, 50], [[0, 1], [2, 3, 4, 5]], list(range(31)))
    assert not md.is_decode and md.max_q_len == 30
    with pytest.raises(ValueError):
        bld.build([1], [100], [[0]], [5])  # table too short
    with pytest.raises(ValueError):
        K8V4AttentionImpl(24, 128, None, 4, kv_cache_dtype="fp8")
    impl = K8V4AttentionImpl(24, 128, None, 4)
    assert abs(impl.scale - 1 / math.sqrt(128)) < 1e-12


def _paged_case(n, q_len, hkv=2, gqa=6, seed=0):
    g = torch.Generator().manual_seed(seed)
    lay = b200_layout(hkv, gqa)
    npg = (n + 15) // 16
    pages = torch.randperm(npg + 3, generator=g)[:npg]
    cache = torch.zeros(npg + 3, lay.page_bytes, dtype=torch.uint8)
    k = torch.randn(n, hkv, 128, generator=g).bfloat16()
    v = torch.randn(n, hkv, 128, generator=g).bfloat16()
    slots = (pages.repeat_interleave(16) * 16 + torch.arange(16).repeat(npg))[:n]
    store_tokens(cache, slots, k, v, lay)
    q = torch.randn(q_len, hkv * gqa, 128, generator=g).bfloat16()
    return lay, cache, pages, q


def test_eager_prefill_matches_oracle_bottom_right():
    n, q_len = 300, 37
    lay, cache, pages, q = _paged_case(n, q_len)
    out = eager_prefill(q, cache, pages, n, lay.hkv, lay.gqa)
    kd, vd = gather_sequence(cache, pages.tolist(), n, lay)
    ends = [n - q_len + t + 1 for t in range(q_len)]
    ref = O.attention_ref(q.float(), kd, vd, ends, lay.gqa, quantize_q=False)
    assert (out - ref).abs().max().item() < 1e-4
    # with the kernels' int8 Q rule
    outq = eager_prefill(q, cache, pages, n, lay.hkv, lay.gqa, quant_q=True)
    refq = O.attention_ref(q.float(), kd, vd, ends, lay.gqa)
    assert (outq - refq).abs().max().item() < 1e-4
    # batched API on CPU
    cu = torch.tensor([0, q_len], dtype=torch.int32)
    bt = pages.view(1, -1).to(torch.int32)
    out2 = paged_prefill(q, cache, bt, torch.tensor([n]), cu, lay.hkv, lay.gqa)
    assert (out2.float() - ref).abs().max().item() < 2e-2


def test_tiled_online_softmax_equals_dense():
    g = torch.Generator().manual_seed(3)
    S = SDPA_MAX_KEYS + 900
    q = torch.randn(3, 6, 128, generator=g)
    k = torch.randn(S, 128, generator=g)
    v = torch.randn(S, 128, generator=g)
    ends = torch.tensor([S - 2, S - 1, S])
    tiled = attention_dense(q, k, v, ends, 1 / math.sqrt(128))
    sc = torch.einsum("tgd,sd->tgs", q, k) / math.sqrt(128)
    sc = sc.masked_fill(torch.arange(S).view(1, 1, -1) >= ends.view(3, 1, 1), float("-inf"))
    ref = torch.einsum("tgs,sd->tgd", torch.softmax(sc, -1), v)
    assert (tiled - ref).abs().max().item() < 1e-4


def test_workspace_sizing_matches_the_native_library():
    """The host's split-K workspace sizes (decode plan, CP exchange slots)
    follow the native kernels' own formula."""
    import pytest
    from k8v4_xpu_b200 import ops
    from k8v4_xpu_b200.attention import plan as P
    from k8v4_xpu_b200.parallel.cp_combine import max_slot_floats
    from k8v4_xpu_b200.runtime.engine import decode_splits
    if not ops.load():
        pytest.skip("native library not built")
    for nseq in (1, 3, 4):
        for hkv in (1, 2, 4):
            for q in (1, 2, 7, 10):
                for gqa in (3, 6):
                    if q * gqa > 64:
                        continue
                    for nsplit in (1, 5, 37, 64):
                        assert P.decode_workspace_floats(nseq, hkv, nsplit, q, gqa) == \
                            ops.decode_ws_floats(nseq, hkv, nsplit, q, gqa)
                    ns = max(2, decode_splits(8192, nseq, hkv))
                    assert ops.decode_ws_floats(nseq, hkv, ns, q, gqa) <= max_slot_floats(nseq, hkv, q, gqa)
