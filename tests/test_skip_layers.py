"""Skip layers: a per-layer fp8 / bf16 KV cache next to the K8/V4 layers (CPU)."""
import math

import pytest
import torch

from k8v4_xpu_b200.kv import skip_layers as S


def test_dtype_resolution_prefers_argument_then_own_env_then_reference_env():
    assert S.resolve_skip_dtype(env={}) == "auto"
    assert S.resolve_skip_dtype(env={"VLLM_KV_SKIP_DTYPE": "fp8"}) == "fp8"
    assert S.resolve_skip_dtype(env={"VLLM_KV_SKIP_DTYPE": "fp8", "K8V4_KV_SKIP_DTYPE": "bfloat16"}) == "bfloat16"
    assert S.resolve_skip_dtype("FP8_E5M2", env={"K8V4_KV_SKIP_DTYPE": "auto"}) == "fp8_e5m2"
    with pytest.raises(ValueError):
        S.resolve_skip_dtype("int4")
    assert S.parse_layers("3, 0,3") == (0, 3)
    assert S.parse_layers(None) == ()
    with pytest.raises(ValueError):
        S.parse_layers([-1])


def test_page_geometry_holds_sixteen_tokens_with_a_16_byte_stride():
    fp8 = S.SkipLayout(4, "fp8")
    bf16 = S.SkipLayout(4, "auto")
    assert fp8.token_bytes == 2 * 4 * 128 and fp8.page_bytes == 16 * 1024
    assert bf16.token_bytes == 2 * 4 * 128 * 2 and bf16.page_bytes == 16 * 2048
    pool = fp8.alloc(5)
    assert pool.shape == (6, fp8.page_bytes) and pool.dtype == torch.uint8
    assert fp8.token_rows(pool).shape == (6 * 16, 1024)
    # capacity unit: two K8/V4 layers of 1234-byte pages and this skip layer
    assert S.pool_bytes_per_page(1234, 3, {2: fp8}) == 2 * 1234 + fp8.page_bytes


@pytest.mark.parametrize("name", ["fp8", "bfloat16", "fp8_e5m2"])
def test_store_roundtrip_and_padding_rows_land_in_the_sink(name):
    torch.manual_seed(0)
    lay = S.SkipLayout(2, name, k_scale=0.5 if name == "fp8" else 1.0)
    pool = lay.alloc(4)
    T = 9
    k = torch.randn(T, 2, 128).bfloat16()
    v = torch.randn(T, 2, 128).bfloat16()
    slots = torch.tensor([3, 17, 40, -1, 63, 0, -1, 21, 8])
    S.store(pool, lay, slots, k, v)
    rows = lay.token_rows(pool)
    kd, vd = lay.decode(rows)
    dt = S.SKIP_DTYPES[name]
    for t, s in enumerate(slots.tolist()):
        if s < 0:
            continue
        ek = (k[t].float() / lay.k_scale).to(dt).float() * lay.k_scale
        ev = (v[t].float() / lay.v_scale).to(dt).float() * lay.v_scale
        assert torch.equal(kd[s], ek) and torch.equal(vd[s], ev)
    written = set(s for s in slots.tolist() if s >= 0)
    untouched = [r for r in range(4 * 16) if r not in written]
    assert int(rows[untouched].abs().sum()) == 0          # only the named slots changed
    assert int(pool[4].abs().sum()) > 0                   # the -1 rows went to the sink page


def _dense(q, k, v, ends, gqa, scale):
    """fp32 per-row causal GQA: q [Tq, hq, D], k/v [S, hkv, D]."""
    Tq, hq, D = q.shape
    out = torch.zeros(Tq, hq, D)
    for t in range(Tq):
        e = int(ends[t])
        if e == 0:
            continue
        for h in range(hq):
            kv = h // gqa
            sc = (q[t, h].float() @ k[:e, kv].T) * scale
            out[t, h] = torch.softmax(sc, -1) @ v[:e, kv]
    return out


def _batch(lay, lens, qlens, gqa, seed=0):
    """Shuffled pages for each sequence, every context token stored; q rows at
    the end of each sequence."""
    g = torch.Generator().manual_seed(seed)
    P = lay.page
    npg = [(n + P - 1) // P for n in lens]
    perm = torch.randperm(sum(npg), generator=g)
    pool = lay.alloc(sum(npg))
    W = max(npg) + 2
    bt = torch.zeros(len(lens), W, dtype=torch.int32)
    ks, vs, off = [], [], 0
    for b, n in enumerate(lens):
        pages = perm[off:off + npg[b]]
        off += npg[b]
        bt[b, :npg[b]] = pages.int()
        bt[b, npg[b]:] = perm[0]  # stale ids past the end
        k = torch.randn(n, lay.hkv, 128, generator=g).bfloat16()
        v = torch.randn(n, lay.hkv, 128, generator=g).bfloat16()
        slots = pages.repeat_interleave(P)[:n] * P + torch.arange(n) % P
        S.store(pool, lay, slots, k, v)
        ks.append(k)
        vs.append(v)
    hq = lay.hkv * gqa
    T = sum(qlens)
    q = torch.randn(T, hq, 128, generator=g).bfloat16()
    cu = torch.tensor([0] + list(torch.tensor(qlens).cumsum(0).tolist()), dtype=torch.int32)
    pos = torch.cat([torch.arange(n - ql, n) for n, ql in zip(lens, qlens)])
    return pool, bt, torch.tensor(lens, dtype=torch.int32), cu, pos, q, ks, vs


@pytest.mark.parametrize("name", ["fp8", "bfloat16"])
@pytest.mark.parametrize("score_bytes", [S.SCORE_TILE_BYTES, 40_000])
def test_paged_attention_matches_dense_causal_gqa(name, score_bytes):
    lay = S.SkipLayout(2, name)
    gqa = 3
    lens, qlens = [37, 5, 70], [7, 1, 33]  # MTP-width rows, a decode row, a prefill chunk
    pool, bt, sl, cu, pos, q, ks, vs = _batch(lay, lens, qlens, gqa)
    out = S.paged_attention(q, pool, lay, bt, sl, cu, pos, max(qlens), gqa, score_bytes=score_bytes)
    assert out.dtype == torch.bfloat16 and out.shape == q.shape
    scale = 1 / math.sqrt(128)
    dt = lay.dtype
    c = cu.tolist()
    for b in range(len(lens)):
        kq = ks[b].float().to(dt).float()
        vq = vs[b].float().to(dt).float()
        ref = _dense(q[c[b]:c[b + 1]].float(), kq, vq, pos[c[b]:c[b + 1]] + 1, gqa, scale)
        assert (out[c[b]:c[b + 1]].float() - ref).abs().max() < 2e-2
        if name == "fp8":  # against unquantized K/V: the fp8 rounding only
            ref16 = _dense(q[c[b]:c[b + 1]].float(), ks[b].float(), vs[b].float(), pos[c[b]:c[b + 1]] + 1, gqa, scale)
            assert (out[c[b]:c[b + 1]].float() - ref16).abs().max() < 0.15


def test_key_tiling_does_not_change_the_result_and_q_ends_override_positions():
    lay = S.SkipLayout(1, "bfloat16")
    lens, qlens = [100, 64], [4, 4]
    pool, bt, sl, cu, pos, q, ks, vs = _batch(lay, lens, qlens, 6, seed=3)
    a = S.paged_attention(q, pool, lay, bt, sl, cu, pos, 4, 6)
    b = S.paged_attention(q, pool, lay, bt, sl, cu, pos, 4, 6, score_bytes=1)  # one page per tile
    assert (a.float() - b.float()).abs().max() < 1e-2
    # a tree: every draft row sees only the context before the drafts plus itself
    ends = torch.tensor([97, 98, 98, 98, 61, 62, 62, 0], dtype=torch.int32)
    c = S.paged_attention(q, pool, lay, bt, sl, cu, pos, 4, 6, q_ends=ends)
    scale = 1 / math.sqrt(128)
    ref0 = _dense(q[:4].float(), ks[0].float(), vs[0].float(), ends[:4], 6, scale)
    ref1 = _dense(q[4:].float(), ks[1].float(), vs[1].float(), ends[4:], 6, scale)
    assert (c[:4].float() - ref0).abs().max() < 2e-2
    assert (c[4:].float() - ref1).abs().max() < 2e-2
    assert torch.equal(c[7], torch.zeros_like(c[7]))  # no visible key -> zero row


def test_rope_rotates_each_half_pair_by_its_position_angle():
    from k8v4_xpu_b200.models.dense import rope_table
    tab = rope_table(64, 128, 10000.0, "cpu")
    x = torch.randn(5, 3, 128).bfloat16()
    pos = torch.tensor([0, 1, 7, 63, 20])
    y = S.apply_rope(x, tab, pos)
    assert torch.equal(y[0], x[0])  # position 0: identity
    ang = 7 * 10000.0 ** (-torch.arange(64, dtype=torch.float64) / 64)  # position 7, pair i
    a, b = x[2].double()[..., :64], x[2].double()[..., 64:]
    want = torch.cat([a * ang.cos() - b * ang.sin(), b * ang.cos() + a * ang.sin()], -1)
    assert (y[2].double() - want).abs().max() < 3e-2
    # rotation keeps each (i, i + 64) pair's norm
    n0 = x.float()[..., :64] ** 2 + x.float()[..., 64:] ** 2
    n1 = y.float()[..., :64] ** 2 + y.float()[..., 64:] ** 2
    assert (n0 - n1).abs().max() < 0.1


def test_engine_config_validates_skip_layers():
    from k8v4_xpu_b200.runtime.engine import EngineConfig
    cfg = EngineConfig(kv_cache_dtype_skip_layers="2,0", kv_skip_dtype="fp8", device="cpu")
    assert cfg.kv_cache_dtype_skip_layers == (0, 2)
    lays = cfg.skip_layouts(3, 4)
    assert sorted(lays) == [0, 2] and lays[0].dtype == torch.float8_e4m3fn and lays[0].hkv == 4
    with pytest.raises(ValueError):
        cfg.skip_layouts(2, 4)  # layer 2 does not hold a cache
    with pytest.raises(ValueError):
        EngineConfig(kv_cache_dtype_skip_layers=(0,), context_parallel_size=2)
    with pytest.raises(ValueError):
        EngineConfig(kv_cache_dtype_skip_layers=(0,), kv_skip_dtype="int4")
    assert EngineConfig().kv_cache_dtype_skip_layers == ()


def test_serve_flags_and_environment():
    from k8v4_xpu_b200 import config as C
    c = C.resolve(["--kv-cache-dtype-skip-layers", "64", "--kv-skip-dtype", "fp8"], env={})
    e = c.engine_config("cpu")
    assert e.kv_cache_dtype_skip_layers == (64,) and e.kv_skip_dtype == "fp8"
    c = C.resolve([], env={"K8V4_KV_SKIP_LAYERS": "1,3", "VLLM_KV_SKIP_DTYPE": "fp8_e5m2"})
    assert c.kv_cache_dtype_skip_layers == (1, 3) and c.kv_skip_dtype == "fp8_e5m2"
    assert C.resolve([], env={}).engine_config("cpu").kv_cache_dtype_skip_layers == ()
    with pytest.raises(ValueError):
        C.resolve(["--kv-cache-dtype-skip-layers", "0", "--context-parallel-size", "2"], env={})


def test_engine_allocates_skip_pools_on_the_shared_page_ids():
    import types
    from k8v4_xpu_b200.kv.layout import b200_layout
    from k8v4_xpu_b200.runtime.engine import EngineConfig, LLMEngine
    lay = b200_layout(2, 6)
    model = types.SimpleNamespace(layers=[None, None], mtp=object(), shape=types.SimpleNamespace(hkv_local=2))
    eng = types.SimpleNamespace(cfg=EngineConfig(kv_cache_dtype_skip_layers=(0, 2), kv_skip_dtype="fp8",
                                                 num_kv_blocks=8, max_model_len=128, device="cpu"),
                                layout=lay, model=model, device=torch.device("cpu"))
    LLMEngine._alloc_cache(eng)
    pages = 8 * (16 // lay.page)
    skip = S.SkipLayout(2, "fp8")
    assert [tuple(c.shape) for c in eng.kv_caches] == [(pages + 1, skip.page_bytes), (pages, lay.page_bytes),
                                                       (pages + 1, skip.page_bytes)]
    assert eng.kv_pool.shape == (1, pages, lay.page_bytes)
    assert sorted(model.skip_kv) == [0, 2]


def test_model_skip_attention_glue_matches_manual_rope_store_attention():
    import types
    from k8v4_xpu_b200.models.config import TINY
    from k8v4_xpu_b200.models.dense import DenseModel, StepInputs, rope_table
    m = DenseModel(TINY, device="cpu")
    m.rope = rope_table(512, 128, TINY.rope_theta, "cpu")
    hq, hkv = m.shape.hq_local, m.shape.hkv_local
    lay = S.SkipLayout(hkv, "fp8")
    torch.manual_seed(1)
    n = 40
    qkv = torch.randn(n, hq + 2 * hkv, 128).bfloat16()
    cache = lay.alloc(4)
    inp = StepInputs(input_ids=torch.zeros(n, dtype=torch.int64), positions=torch.arange(n),
                     slots=torch.arange(n) + 16, cu_q=torch.tensor([0, n], dtype=torch.int32),
                     seq_lens=torch.tensor([n], dtype=torch.int32),
                     block_table=torch.tensor([[1, 2, 3]], dtype=torch.int32),
                     logit_rows=torch.tensor([n - 1]), max_q_len=n, is_decode=False)
    out = m._skip_attention(qkv, inp, cache, lay)
    q = S.apply_rope(qkv[:, :hq], m.rope, inp.positions)
    k = S.apply_rope(qkv[:, hq:hq + hkv], m.rope, inp.positions).float().to(lay.dtype).float()
    v = qkv[:, hq + hkv:].float().to(lay.dtype).float()
    ref = _dense(q.float(), k, v, inp.positions + 1, m.shape.gqa_local, 1 / math.sqrt(128))
    assert (out.float() - ref).abs().max() < 2e-2
    assert int(cache[0].abs().sum()) == 0  # page 0 is not in the table and was not written
