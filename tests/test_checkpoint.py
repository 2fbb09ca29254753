"""Checkpoint round trip, TP shard loading, embedding shards, GPTQ bake (CPU)."""
import json

import pytest
import torch

from k8v4_xpu_b200.models import gptq
from k8v4_xpu_b200.models.checkpoint import load_checkpoint, read_model_config, save_checkpoint
from k8v4_xpu_b200.models.config import TINY
from k8v4_xpu_b200.models.dense import DenseModel
from k8v4_xpu_b200.tools import bake


def _model(tp=1, rank=0, seed=5):
    return DenseModel(TINY, tp=tp, rank=rank, device="cpu").random_init(seed=seed)


def test_save_load_roundtrip_exact(tmp_path):
    m = _model()
    m.init_mtp(seed=2)
    save_checkpoint(m, str(tmp_path))
    assert read_model_config(str(tmp_path)) == TINY.__class__(**{**TINY.__dict__})
    m2 = DenseModel(TINY, device="cpu")
    m2.mtp = None
    load_checkpoint(m2, str(tmp_path))
    for a, b in zip(m.layers, m2.layers):
        for f in ("qkv", "o", "gate_up", "down"):
            assert torch.equal(getattr(a, f).qweight, getattr(b, f).qweight)
            assert torch.equal(getattr(a, f).scales, getattr(b, f).scales)
        assert torch.equal(a.input_norm, b.input_norm)
    assert torch.equal(m.embed_codes, m2.embed_codes) and torch.equal(m.embed_scales, m2.embed_scales)
    assert torch.equal(m.lm_head.weight, m2.lm_head.weight)
    assert m2.mtp is not None and torch.equal(m.mtp.eh_proj.qweight, m2.mtp.eh_proj.qweight)
    assert bake.verify_checkpoint(str(tmp_path))["linears"] == 7 * TINY.num_layers


def test_tp_loading_matches_tp_random_init(tmp_path):
    full = _model(seed=9)
    save_checkpoint(full, str(tmp_path))
    for rank in range(2):
        ref = _model(tp=2, rank=rank, seed=9)       # random_init shards the same full draws
        m = DenseModel(TINY, tp=2, rank=rank, device="cpu")
        load_checkpoint(m, str(tmp_path))
        for a, b in zip(ref.layers, m.layers):
            for f in ("qkv", "o", "gate_up", "down"):
                assert torch.equal(getattr(a, f).qweight, getattr(b, f).qweight), (rank, f)
        assert torch.equal(ref.embed_codes, m.embed_codes)  # only this rank's vocab rows
        assert m.embed_codes.shape[0] == TINY.vocab // 2
        assert torch.equal(ref.lm_head.weight, m.lm_head.weight)


def test_embedding_vocab_shards_sum_to_full_lookup():
    """Behaviour of the reference's embedding TP fixture: each rank holds its
    vocab rows; ids outside a shard embed to zero; the ranks' sum is the full
    lookup."""
    V, H = 1000, 64
    w = torch.randn(V, H)
    codes, scales = gptq.quantize_int8_rows(w)
    ids = torch.tensor([0, 499, 500, 999, 123])
    full = codes[ids].float() * scales[ids].float()
    tot = torch.zeros(len(ids), H)
    tp = 2
    for r in range(tp):
        lo, hi = r * V // tp, (r + 1) * V // tp
        local = ids - lo
        inside = (local >= 0) & (local < hi - lo)
        rows = codes[lo:hi][local.clamp(0, hi - lo - 1)].float() * scales[lo:hi][local.clamp(0, hi - lo - 1)].float()
        tot += torch.where(inside.view(-1, 1), rows, torch.zeros_like(rows))
    assert torch.equal(tot, full)


def test_gptq_beats_rtn_on_correlated_inputs():
    g = torch.Generator().manual_seed(0)
    K, N, n = 256, 64, 2048
    base = torch.randn(n, 8, generator=g)
    x = base @ torch.randn(8, K, generator=g) + 0.05 * torch.randn(n, K, generator=g)  # low-rank inputs
    w = torch.randn(K, N, generator=g) * 0.05
    acc = bake.HessianAccumulator(K)
    for chunk in x.split(512):
        acc.add(chunk)
    assert torch.allclose(acc.H, 2 * x.double().t() @ x.double() / n, rtol=1e-6, atol=1e-8)
    c_rtn, s_rtn = bake.gptq_quantize(w)
    c_q, s_q = bake.gptq_quantize(w, acc.H)
    deq = lambda c, s: (c.float() - 8).view(K // 128, 128, N) * s.view(K // 128, 1, N)  # noqa: E731
    ref = x @ w
    err_rtn = ((x @ deq(c_rtn, s_rtn).view(K, N)) - ref).pow(2).mean()
    err_q = ((x @ deq(c_q, s_q).view(K, N)) - ref).pow(2).mean()
    assert err_q < 0.7 * err_rtn, (float(err_q), float(err_rtn))
    assert c_q.max() <= 15 and s_q.dtype == torch.float32


def test_bake_dense_checkpoint(tmp_path):
    from safetensors.torch import save_file
    from k8v4_xpu_b200.models.checkpoint import config_to_hf
    src, out = tmp_path / "dense", tmp_path / "gptq"
    src.mkdir()
    cfg = TINY.__class__(**{**TINY.__dict__, "num_layers": 1})
    hf = config_to_hf(cfg)
    hf.pop("quantization_config")
    (src / "config.json").write_text(json.dumps(hf))
    g = torch.Generator().manual_seed(1)
    t = {}
    H, I = cfg.hidden, cfg.intermediate
    dims = {"self_attn.q_proj": (cfg.q_size, H), "self_attn.k_proj": (cfg.kv_size, H),
            "self_attn.v_proj": (cfg.kv_size, H), "self_attn.o_proj": (H, cfg.q_size),
            "mlp.gate_proj": (I, H), "mlp.up_proj": (I, H), "mlp.down_proj": (H, I)}
    for lin, shape in dims.items():
        t["model.layers.0.%s.weight" % lin] = (torch.randn(*shape, generator=g) * 0.02).bfloat16()
    for nm in ("input_layernorm", "post_attention_layernorm"):
        t["model.layers.0.%s.weight" % nm] = torch.ones(H).bfloat16()
    t["model.norm.weight"] = torch.ones(H).bfloat16()
    t["model.embed_tokens.weight"] = (torch.randn(cfg.vocab, H, generator=g) * 0.02).bfloat16()
    save_file(t, str(src / "model.safetensors"))
    rep = bake.bake_dense(str(src), str(out))
    assert rep == {"linears_gptq": 0, "linears_rtn": 7, "layers": 1}
    assert bake.verify_checkpoint(str(out))["linears"] == 7
    m = DenseModel(cfg, device="cpu")
    load_checkpoint(m, str(out))
    w = t["model.layers.0.mlp.down_proj.weight"].float().t()
    deq = gptq.dequant_int4(m.layers[0].down.qweight, m.layers[0].down.scales)
    assert (deq - w).abs().max() <= m.layers[0].down.scales.float().max() * 0.5 + 1e-3
    with pytest.raises(ValueError):
        load_checkpoint(DenseModel(TINY.__class__(**{**TINY.__dict__, "hidden": 1024}), device="cpu"), str(out))


def test_bake_cli_random_and_verify(tmp_path):
    import subprocess
    import sys
    out = subprocess.run([sys.executable, "-m", "k8v4_xpu_b200.tools.bake", "random", "--preset", "tiny",
                          "--layers", "1", "--out", str(tmp_path / "ck")], capture_output=True, text=True,
                         timeout=300)
    assert out.returncode == 0, out.stderr
    rep = json.loads(out.stdout.strip().splitlines()[-1])
    assert rep["layers"] == 1 and rep["mtp"] and rep["lm_head_rows"] == TINY.vocab


def test_tp8_shards_replicate_kv_heads_and_tile_the_full_model():
    """TP 8 on the 27B head structure (24 Q heads, 4 KV heads): every rank
    holds 3 Q heads and KV head rank // 2 (two ranks per KV head), and the
    ranks' shards are exact slices of the TP 1 weights."""
    from k8v4_xpu_b200.models.config import ModelConfig
    cfg = ModelConfig(name="tp8-shape", num_layers=1, hidden=512, num_heads=24, num_kv_heads=4, head_dim=128,
                      intermediate=2048, vocab=4096, max_position=1024)
    D = cfg.head_dim
    full = DenseModel(cfg, device="cpu").random_init(seed=11)
    F = full.layers[0]
    fq = F.qkv.dense_t()            # [K, q | k | v]
    fo, fg, fd = F.o.dense_t(), F.gate_up.dense_t(), F.down.dense_t()
    q_sz, kv_sz, I = cfg.q_size, cfg.kv_size, cfg.intermediate
    for rank in range(8):
        m = DenseModel(cfg, tp=8, rank=rank, device="cpu").random_init(seed=11)
        sh = m.shape
        assert (sh.hq_local, sh.hkv_local, sh.kv_replicas, sh.gqa_local) == (3, 1, 2, 3)
        L = m.layers[0]
        kvh = rank // 2
        want_qkv = torch.cat([fq[:, rank * 3 * D:(rank + 1) * 3 * D],
                              fq[:, q_sz + kvh * D:q_sz + (kvh + 1) * D],
                              fq[:, q_sz + kv_sz + kvh * D:q_sz + kv_sz + (kvh + 1) * D]], 1)
        assert torch.equal(L.qkv.dense_t(), want_qkv), rank
        assert torch.equal(L.o.dense_t(), fo[rank * 3 * D:(rank + 1) * 3 * D]), rank
        il = I // 8
        assert torch.equal(L.gate_up.dense_t(), torch.cat([fg[:, rank * il:(rank + 1) * il],
                                                           fg[:, I + rank * il:I + (rank + 1) * il]], 1)), rank
        assert torch.equal(L.down.dense_t(), fd[rank * il:(rank + 1) * il]), rank
        v = cfg.vocab // 8
        assert torch.equal(m.lm_head.weight[:v], full.lm_head.weight[rank * v:(rank + 1) * v]), rank
        assert torch.equal(m.embed_codes, full.embed_codes[rank * v:(rank + 1) * v]), rank


def test_checkpoint_files_are_written_atomically_config_last(tmp_path, monkeypatch):
    """A save that dies part way leaves no file under its final name and no
    config.json (the marker of a complete directory)."""
    import os
    from k8v4_xpu_b200.models import checkpoint as C
    m = _model()
    real = C._save
    calls = []

    def dying(tensors, path):
        calls.append(path)
        if path.endswith(C.SIDE_FILE):
            raise OSError("disk full")
        real(tensors, path)

    monkeypatch.setattr(C, "_save", dying)
    with pytest.raises(OSError):
        save_checkpoint(m, str(tmp_path / "a"))
    names = set(os.listdir(tmp_path / "a"))
    assert "config.json" not in names and C.SIDE_FILE not in names
    assert not any(n.endswith(".partial") for n in names)
    monkeypatch.setattr(C, "_save", real)
    save_checkpoint(m, str(tmp_path / "b"))
    names = set(os.listdir(tmp_path / "b"))
    assert "config.json" in names and C.SIDE_FILE in names
    assert not any(n.endswith(".partial") for n in names)


def test_27b_shards_meet_the_kernels_tiling_at_every_tp():
    """The headline model's per-rank shapes at TP 1/2/4/8 fit the GEMMs'
    128-wide feature and k tiles (the lm_head pads its vocab shard), the
    decode kernels' head layout, and the sequence-parallel prefill: every
    chunk of the 128,197-token benchmark prompt gives every rank a tile."""
    from k8v4_xpu_b200.models.config import DENSE_27B, TPShape
    from k8v4_xpu_b200.parallel.seq_parallel import TILE, SeqParallel, owned_rows, tile_owners
    cfg = DENSE_27B
    D, H = cfg.head_dim, cfg.hidden
    ctx, chunk = 128197, 4224
    chunks = [min(chunk, ctx - s) for s in range(0, ctx, chunk)]
    for tp in (1, 2, 4, 8):
        sh = TPShape.make(cfg, tp)
        gemms = {"qkv": ((sh.hq_local + 2 * sh.hkv_local) * D, H), "o": (H, sh.hq_local * D),
                 "gate_up": (2 * sh.inter_local, H), "down": (H, sh.inter_local)}
        for name, (n, k) in gemms.items():
            assert n % 128 == 0 and k % 128 == 0, (tp, name, n, k)
        assert sh.hkv_local >= 1 and sh.gqa_local * 7 <= 64  # MTP verify rows per KV head in one decode tile
        assert H % 64 == 0 and sh.vocab_local % 8 == 0       # cluster norm slices, argmax vector loads
        if tp > 1:
            sp = object.__new__(SeqParallel)
            sp.world, sp.max_rows, sp.hidden = tp, chunk, H
            for rows in chunks:
                assert sp.fits(rows, H), (tp, rows)
                t0 = tile_owners(rows, tp)
                assert all(owned_rows(rows, t0, o)[1] > 0 for o in range(tp)), (tp, rows)
            assert TILE * tp <= min(chunks)
