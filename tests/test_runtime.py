"""Block manager, prefix cache, scheduler, GPTQ format, TP shapes, path policy (CPU)."""
import random

import pytest
import torch

from k8v4_xpu_b200.layers import linear as LIN
from k8v4_xpu_b200.models import gptq
from k8v4_xpu_b200.models.config import DENSE_27B, TINY, ModelConfig, TPShape
from k8v4_xpu_b200.runtime.block_manager import BlockManager, CapacityError, chain_hash
from k8v4_xpu_b200.runtime.scheduler import SamplingParams, Scheduler


# ---------------------------------------------------------------- blocks
def test_block_manager_alloc_grow_free():
    bm = BlockManager(8, block_size=32, page=16)
    assert bm.ratio == 2
    assert bm.allocate(0, list(range(40))) == 0
    bm.ensure(0, 40)
    assert len(bm.tables[0]) == 2
    assert bm.page_table(0) == [p for b in bm.tables[0] for p in (2 * b, 2 * b + 1)]
    b1 = bm.tables[0][1]
    assert bm.slot(0, 33) == b1 * 32 + 1
    bm.check_invariants()
    bm.free_seq(0)
    assert bm.num_free == 8
    bm.check_invariants()
    with pytest.raises(ValueError):
        BlockManager(4, block_size=24, page=16)


def test_capacity_error_is_raised_not_silent():
    bm = BlockManager(2, block_size=16)
    bm.allocate(0, list(range(10)))
    bm.ensure(0, 32)
    with pytest.raises(CapacityError):
        bm.allocate(1, list(range(20)))
    with pytest.raises(CapacityError):
        bm.ensure(0, 33)
    bm.check_invariants()


def test_prefix_cache_hit_share_and_evict():
    bm = BlockManager(6, block_size=16)
    prompt = list(range(50))
    bm.allocate(0, prompt)
    bm.ensure(0, 50)
    bm.publish(0, prompt, 50)
    assert len(bm.cached) == 3
    # a second prompt sharing 40 tokens reuses the first two full blocks
    p2 = prompt[:40] + [999] * 5
    assert bm.allocate(1, p2) == 32
    assert bm.tables[1][:2] == bm.tables[0][:2]
    assert bm.info[bm.tables[0][0]].ref == 2
    bm.check_invariants()
    # the whole prompt never matches: the last token must be computed
    blocks, _ = bm.match_prefix(prompt[:48])
    assert len(blocks) == 2
    bm.free_seq(0)
    bm.free_seq(1)
    assert bm.num_free == 6 and len(bm.evictable) == 3
    # allocating beyond the free list evicts the LRU cached blocks
    bm.allocate(2, list(range(1000, 1090)))
    bm.ensure(2, 90)
    assert len(bm.cached) == 0
    bm.check_invariants()


def test_publish_deduplicates_identical_blocks():
    bm = BlockManager(8, block_size=16)
    p = list(range(33))
    for s in (0, 1):
        bm.allocate(s, p, prefix=False)
        bm.ensure(s, 33)
    bm.publish(0, p, 33)
    bm.publish(1, p, 33)
    assert bm.tables[0][:2] == bm.tables[1][:2]
    bm.check_invariants()


def test_truncate_and_fork_copy_on_write():
    bm = BlockManager(10, block_size=16)
    p = list(range(40))
    bm.allocate(0, p)
    bm.ensure(0, 47)   # 40 tokens + 7 speculative slots
    bm.truncate(0, 41)  # rollback after verify
    assert len(bm.tables[0]) == 3
    copies = bm.fork(0, 1, 41)
    assert bm.tables[1][:2] == bm.tables[0][:2]
    assert copies == [(bm.tables[0][2], bm.tables[1][2])]
    bm.check_invariants()
    bm.truncate(0, 16)
    assert len(bm.tables[0]) == 1
    bm.check_invariants()


def test_chain_hash_depends_on_parent():
    a = chain_hash(None, [1, 2, 3])
    assert chain_hash(a, [4]) != chain_hash(None, [4])
    assert chain_hash(None, [1, 2, 3]) == a


def test_block_manager_random_ops_keep_invariants():
    rng = random.Random(0)
    bm = BlockManager(40, block_size=16)
    live = {}
    nxt = 0
    for _ in range(400):
        op = rng.random()
        if op < 0.4:
            base = rng.choice([0, 1000, 2000])
            toks = list(range(base, base + rng.randint(1, 100)))
            try:
                bm.allocate(nxt, toks)
                bm.ensure(nxt, len(toks))
                bm.publish(nxt, toks, len(toks))
                live[nxt] = len(toks)
            except CapacityError:
                bm.free_seq(nxt)
            nxt += 1
        elif op < 0.6 and live:
            s = rng.choice(list(live))
            bm.free_seq(s)
            del live[s]
        elif op < 0.8 and live:
            s = rng.choice(list(live))
            n = max(1, live[s] - rng.randint(0, 10))
            bm.truncate(s, n)
            live[s] = n
        elif live:
            s = rng.choice(list(live))
            try:
                bm.ensure(s, live[s] + 7)
                live[s] += 7
            except CapacityError:
                pass
        bm.check_invariants()


# ------------------------------------------------------------- scheduler
def test_scheduler_chunked_prefill_then_decode_first():
    bm = BlockManager(2000, block_size=16)
    sch = Scheduler(bm, max_num_seqs=4, max_num_batched_tokens=4224)
    a = sch.add(list(range(10000)), SamplingParams(max_tokens=4))
    out = sch.schedule()
    assert [c.num_tokens for c in out.chunks] == [4224] and not out.chunks[0].needs_logits
    a.computed += 4224
    out = sch.schedule()
    assert out.chunks[0].start == 4224 and out.chunks[0].num_tokens == 4224
    a.computed += 4224
    b = sch.add(list(range(500)), SamplingParams(max_tokens=4))
    out = sch.schedule()
    assert [(c.seq.seq_id, c.num_tokens, c.needs_logits) for c in out.chunks] == [
        (a.seq_id, 10000 - 8448, True), (b.seq_id, 500, True)]
    a.computed = 10000
    a.output.append(1)
    b.computed = 500
    b.output.append(2)
    out = sch.schedule()
    assert out.is_decode_only and [c.num_tokens for c in out.chunks] == [1, 1]
    # MTP width: 1 + drafts
    a.draft = [5] * 6
    out = sch.schedule()
    assert [c.num_tokens for c in out.chunks] == [7, 1]


def test_scheduler_limits_and_preemption():
    bm = BlockManager(5, block_size=16)  # 80 tokens: one max_model_len sequence fits the pool
    sch = Scheduler(bm, max_num_seqs=2, max_num_batched_tokens=64, max_model_len=80)
    with pytest.raises(ValueError):
        sch.add([])
    with pytest.raises(ValueError):
        sch.add(list(range(70)), SamplingParams(max_tokens=20))
    a = sch.add(list(range(40)), SamplingParams(max_tokens=40))
    b = sch.add(list(range(100, 110)))
    out = sch.schedule()
    assert [c.seq for c in out.chunks] == [a, b]
    a.output = [7] * 25  # 65 tokens, 64 written: the next write needs two more blocks, one is free
    a.computed = 64
    b.output = [1]
    b.computed = 10
    out = sch.schedule()
    assert out.preempted == [a] and sch.num_preemptions == 1
    # recompute preemption keeps prompt and output (max_tokens counts the output)
    assert len(a.prompt) == 40 and a.output == [7] * 25 and a.computed == 0
    assert a.prefill_target == 65 and a.in_prefill
    assert [c.seq for c in out.chunks] == [b]
    bm.check_invariants()
    sch.finish(b, "length")
    out = sch.schedule()  # readmitted: prefill every token it held, in budget-sized chunks
    assert [(c.seq, c.start, c.num_tokens, c.is_prefill, c.needs_logits) for c in out.chunks] == [(a, 0, 64, True, False)]
    a.computed = 64
    out = sch.schedule()
    assert [(c.start, c.num_tokens, c.needs_logits) for c in out.chunks] == [(64, 1, True)]
    a.computed = 65
    a.output.append(8)  # sampled from the recompute prefill's last row
    assert not a.in_prefill
    out = sch.schedule()
    assert [(c.start, c.num_tokens, c.is_prefill) for c in out.chunks] == [(65, 1, False)]
    bm.check_invariants()


# ------------------------------------------------------------------ GPTQ
def test_gptq_pack_roundtrip_and_layout():
    g = torch.Generator().manual_seed(0)
    w = torch.randn(256, 24, generator=g)
    codes, scales = gptq.quantize_int4_rtn(w)
    packed = gptq.pack_int4(codes, scales)
    q = packed["qweight"]
    assert q.dtype == torch.int32 and q.shape == (32, 24)
    assert packed["scales"].shape == (2, 24) and packed["scales"].dtype == torch.float16
    assert (packed["qzeros"] == 0x77777777).all() if "qzeros" in packed else True
    assert torch.equal(gptq.unpack_int4(q), codes)
    # row k lives in word k//8 at nibble k%8 (low nibble first)
    assert int(q[0, 0]) & 0xF == int(codes[0, 0])
    assert (int(q[0, 0]) >> 4) & 0xF == int(codes[1, 0])
    deq = gptq.dequant_int4(q, packed["scales"])
    assert (deq - w).abs().max() <= packed["scales"].float().max() * 0.5 + 1e-3


def test_quant_refs_agree():
    g = torch.Generator().manual_seed(1)
    x = torch.randn(5, 256, generator=g)
    w = torch.randn(256, 64, generator=g)
    codes, scales = gptq.quantize_int4_rtn(w)
    p = gptq.pack_int4(codes, scales)
    y16 = gptq.w4a16_ref(x.bfloat16(), p["qweight"], p["scales"])
    xq, xs = gptq.quant_act_rows(x.bfloat16())
    y8 = gptq.w4a8_ref(xq, xs, p["qweight"], p["scales"])
    ref = x @ gptq.dequant_int4(p["qweight"], p["scales"])
    assert (y16.float() - ref).abs().max() < 0.05 * ref.abs().max()
    assert (y8.float() - ref).abs().max() < 0.05 * ref.abs().max()
    wq, ws = gptq.quantize_int8_rows(w.t().contiguous())
    y88 = gptq.w8a8_ref(xq, xs, wq, ws)
    assert (y88.float() - x @ w).abs().max() < 0.05 * (x @ w).abs().max()


# -------------------------------------------------------- config / policy
def test_tp_shapes():
    assert DENSE_27B.gqa == 6 and DENSE_27B.q_size == 3072
    s1 = TPShape.make(DENSE_27B, 1)
    assert (s1.hq_local, s1.hkv_local, s1.gqa_local) == (24, 4, 6)
    s4 = TPShape.make(DENSE_27B, 4)
    assert (s4.hq_local, s4.hkv_local, s4.inter_local) == (6, 1, 4352)
    s8 = TPShape.make(DENSE_27B, 8)
    assert (s8.hq_local, s8.hkv_local, s8.kv_replicas, s8.gqa_local) == (3, 1, 2, 3)
    assert s8.kv_heads_of(5, 4) == [2]
    assert s4.kv_heads_of(3, 4) == [3]
    with pytest.raises(ValueError):
        TPShape.make(DENSE_27B, 5)
    with pytest.raises(ValueError):
        ModelConfig(num_heads=10, num_kv_heads=4)
    assert ModelConfig.from_dict({**DENSE_27B.__dict__, "extra": 1}) == DENSE_27B
    assert TINY.tp_shard(2).hq_local == 6


def test_w4a8_gate_matches_reference_rule(monkeypatch):
    assert LIN.uses_w4a8("model.layers.3.mlp.down_proj", 129)
    assert not LIN.uses_w4a8("model.layers.3.mlp.down_proj", 128)
    assert not LIN.uses_w4a8("model.layers.3.self_attn.qkv_proj", 4224)
    assert not LIN.uses_w4a8("model.layers.3.mlp.gate_up_proj", 4224, enabled=False)
    monkeypatch.setenv("K8V4_PREFILL_GEMM", "w4a16")
    assert not LIN.w4a8_enabled()
    monkeypatch.setenv("K8V4_PREFILL_GEMM", "bogus")
    with pytest.raises(ValueError):
        LIN.w4a8_enabled()
    monkeypatch.delenv("K8V4_PREFILL_GEMM")
    assert LIN.w4a8_enabled()


def test_split_k_policy_fills_the_gpu():
    assert LIN.split_for(1, 6144, 5120) == 1 or LIN.split_for(1, 6144, 5120) * 48 <= 148
    assert LIN.split_for(200, 6144, 5120) == 1
    s = LIN.split_for(1, 5120, 17408)
    assert 1 < s and s * 40 <= 148 and (17408 // 128) // s >= 4


def test_gemm_diagnostics_log_each_branch_once(caplog):
    import logging
    from k8v4_xpu_b200.layers import linear
    linear._NOTED.clear()
    env = {"K8V4_GEMM_DIAGNOSTICS": "1"}
    with caplog.at_level(logging.INFO, logger="k8v4"):
        linear.note_gemm_branch("layers.0.mlp.gate_up", 4224, "w4a8", env)
        linear.note_gemm_branch("layers.0.mlp.gate_up", 2000, "w4a8", env)
        linear.note_gemm_branch("layers.0.mlp.gate_up", 1, "w4a16", env)
        linear.note_gemm_branch("layers.1.mlp.gate_up", 1, "w4a16", {})  # switch off: nothing
    msgs = [r.getMessage() for r in caplog.records if r.name == "k8v4"]
    assert msgs == ["gemm layers.0.mlp.gate_up: w4a8 (first at 4224 rows)",
                    "gemm layers.0.mlp.gate_up: w4a16 (first at 1 rows)"]


def test_token_view_matches_list_concatenation():
    import random
    from k8v4_xpu_b200.runtime.scheduler import TokenView
    rng = random.Random(0)
    for _ in range(2000):
        a = [rng.randrange(100) for _ in range(rng.randrange(0, 6))]
        b = [rng.randrange(100) for _ in range(rng.randrange(0, 6))]
        v, ref = TokenView(a, b), a + b
        assert len(v) == len(ref) and list(v) == ref
        i = rng.randrange(-len(ref) - 2, len(ref) + 2)
        if -len(ref) <= i < len(ref):
            assert v[i] == ref[i]
        else:
            with pytest.raises(IndexError):
                v[i]
        s = slice(rng.choice([None] + list(range(-8, 9))), rng.choice([None] + list(range(-8, 9))),
                  rng.choice([None, 1, 2, -1]))
        assert list(v[s]) == ref[s]


def test_block_manager_keeps_no_state_for_finished_sequences():
    bm = BlockManager(64, block_size=16)
    seen = set()
    for sid in range(500):
        bm.allocate(sid, list(range(sid % 7, sid % 7 + 40)))
        bm.ensure(sid, 40)
        seen.add(bm.version[sid])
        bm.free_seq(sid)
    assert bm.version == {} and bm.tables == {} and bm.keys == {}
    # a sequence allocated again (after a preemption) gets a version it never had
    bm.allocate(7, [1, 2, 3])
    assert bm.version[7] not in seen
    bm.check_invariants()


def test_engine_fork_and_private_clone_copy_the_kv_pages():
    """``fork_sequence`` shares the parent's full blocks and copies its tail
    block's pages in every layer; ``clone_sequence_private`` copies every
    written page into blocks of its own. The engine's host logic runs on CPU
    tensors standing in for the KV pools."""
    import types
    from k8v4_xpu_b200.runtime.engine import LLMEngine
    page, block, page_bytes = 16, 32, 8
    eng = object.__new__(LLMEngine)  # host logic only (no model, no GPU)
    eng.device = torch.device("cpu")
    eng.blocks = BlockManager(12, block_size=block, page=page, enable_prefix_caching=False)
    eng.scheduler = Scheduler(eng.blocks, 4, 256, 1, 4096)
    eng.layout = types.SimpleNamespace(page=page)
    ratio = block // page
    eng.kv_caches = [torch.zeros((12 * ratio, page_bytes), dtype=torch.uint8) for _ in range(2)]
    seq = eng.add_request(list(range(70)), SamplingParams(max_tokens=8))
    eng.scheduler.schedule()
    seq.computed = 70
    for li, layer in enumerate(eng.kv_caches):  # every page of the pools carries its id and layer
        layer.copy_((torch.arange(layer.shape[0]).view(-1, 1) * 3 + li).to(torch.uint8).expand_as(layer))
    parent = list(eng.blocks.tables[seq.seq_id])
    assert len(parent) == 3  # 70 tokens in 32-token blocks: two full, one partial

    child = eng.fork_sequence(seq)
    ct = eng.blocks.tables[child.seq_id]
    assert ct[:2] == parent[:2] and ct[2] != parent[2]
    assert child.computed == 70 and child in eng.scheduler.running
    for layer in eng.kv_caches:
        src, dst = parent[2], ct[2]
        assert torch.equal(layer[dst * ratio:(dst + 1) * ratio], layer[src * ratio:(src + 1) * ratio])

    clone = eng.clone_sequence_private(seq)
    cp_pages = eng.blocks.page_table(clone.seq_id)
    pp = eng.blocks.page_table(seq.seq_id)
    n = (70 + page - 1) // page
    assert not set(cp_pages[:n]) & set(pp[:n])  # nothing shared
    for layer in eng.kv_caches:
        assert torch.equal(layer[cp_pages[:n]], layer[pp[:n]])
    assert clone.computed == 70 and clone.prompt == seq.prompt
    eng.blocks.check_invariants()
