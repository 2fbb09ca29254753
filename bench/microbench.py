#!/usr/bin/env python3
"""Per-kernel microbenchmarks at the 27B decoder's shapes, with roofline fractions.

Each kernel is timed with CUDA events on its stream after warm-up, with an
L2 flush (a 256 MB write) between iterations so weights and KV come from
HBM. Fractions are against MEASURED_PEAKS.json (STREAM copy GB/s and cuBLAS
bf16 TFLOP/s) when present, else the pool's fallback (6,650 GB/s, 1,590 TF).

    python bench/microbench.py [--only gemm|mlp|attn|attnlib|misc] [--ctx 128197]
"""
from __future__ import annotations

import argparse
import json
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import torch  # noqa: E402

from k8v4_xpu_b200 import ops  # noqa: E402
from k8v4_xpu_b200.kv.layout import b200_layout  # noqa: E402
from k8v4_xpu_b200.layers.linear import split_for  # noqa: E402


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, "fallback"


HBM, TF, SRC = peaks()
_flush = None


def timeit(fn, iters=20, warmup=3, graph=True):
    """Median device time of ``fn``: captured in a CUDA graph and replayed
    after an L2-flushing write, so neither host launch latency nor cached
    weights enter the number."""
    global _flush
    if _flush is None:
        _flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    run = fn
    if graph:
        g = torch.cuda.CUDAGraph()
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            fn()
        torch.cuda.current_stream().wait_stream(s)
        with torch.cuda.graph(g, stream=s):
            fn()
        run = g.replay
    evs = []
    for _ in range(iters):
        _flush.fill_(1)  # keeps the GPU busy while the host queues the next replay
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        run()
        b.record()
        evs.append((a, b))
    torch.cuda.synchronize()
    ts = sorted(a.elapsed_time(b) / 1e3 for a, b in evs)
    return ts[len(ts) // 2]


def rand_int4(N, K):
    qw = torch.randint(-2**31, 2**31 - 1, (K // 8, N), dtype=torch.int32, device="cuda")
    sc = (torch.rand(K // 128, N, device="cuda") * 0.01 + 0.001).half()
    return qw, sc


def report(name, sec, bytes_=None, flops=None, **kw):
    row = {"kernel": name, "us": round(sec * 1e6, 2)}
    if bytes_:
        gbs = bytes_ / sec / 1e9
        row.update(gbs=round(gbs, 1), hbm_frac=round(gbs / HBM, 3))
    if flops:
        tf = flops / sec / 1e12
        row.update(tflops=round(tf, 1), bf16_frac=round(tf / TF, 3))
    row.update(kw)
    print(json.dumps(row), flush=True)
    return row


def bench_gemm():
    H, I, Q, KV, V = 5120, 17408, 3072, 512, 151936
    shapes = {"qkv": (Q + 2 * KV, H), "o": (H, Q), "gate_up": (2 * I, H), "down": (H, I)}
    ws = torch.zeros(64 * 2 * I, dtype=torch.float32, device="cuda")
    for name, (N, K) in shapes.items():
        qw, sc = rand_int4(N, K)
        wbytes = qw.numel() * 4 + sc.numel() * 2
        for M in (1, 4, 7, 28):
            x = torch.randn(M, K, device="cuda").bfloat16()
            split = split_for(M, N, K)
            out = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
            t = timeit(lambda: ops.wq_gemm(ops.W4A16, qw, sc, x, out=out, ws=ws, split=split))
            report("w4a16 %s M=%d" % (name, M), t, bytes_=wbytes, flops=2 * M * N * K, split=split)
        for mode, label in ((ops.W4A16, "w4a16"), (ops.W4A8, "w4a8")):
            M = 4224
            if mode == ops.W4A16:
                x = torch.randn(M, K, device="cuda").bfloat16()
                t = timeit(lambda: ops.wq_gemm(mode, qw, sc, x), iters=10)
            else:
                xq = torch.randint(-127, 127, (M, K), dtype=torch.int8, device="cuda")
                xs = torch.rand(M, device="cuda") * 0.01
                t = timeit(lambda: ops.wq_gemm(mode, qw, sc, xq, xscale=xs), iters=10)
            report("%s %s M=%d" % (label, name, M), t, flops=2 * M * N * K)
    # lm_head (int8 rows, int8 tokens)
    w8 = torch.randint(-127, 127, (V, H), dtype=torch.int8, device="cuda")
    s8 = (torch.rand(V, device="cuda") * 0.01).half()
    for M in (1, 4):
        xq = torch.randint(-127, 127, (M, H), dtype=torch.int8, device="cuda")
        xs = torch.rand(M, device="cuda") * 0.01
        t = timeit(lambda: ops.wq_gemm(ops.W8A8, w8, s8, xq, xscale=xs))
        report("w8a8 lm_head M=%d" % M, t, bytes_=V * H + V * 2)


def bench_mlp():
    """BASELINE config 2 at TP1: the W4A8 MLP layer (int8 activations with a
    per-token scale; gate_up -> SiLU-mul + int8 quant -> down) at M = 1, 7,
    28, 4224 and 16384 tokens; each GEMM and the whole layer."""
    H, I = 5120, 17408
    gq, gs = rand_int4(2 * I, H)
    dq, ds = rand_int4(H, I)
    for M in (1, 7, 28, 4224, 16384):
        xq = torch.randint(-127, 127, (M, H), dtype=torch.int8, device="cuda")
        xs = torch.rand(M, device="cuda") * 0.01
        gu = torch.empty(M, 2 * I, dtype=torch.bfloat16, device="cuda")
        out = torch.empty(M, H, dtype=torch.bfloat16, device="cuda")
        aq, as_ = ops.silu_mul(ops.wq_gemm(ops.W4A8, gq, gs, xq, xscale=xs, out=gu), quant=True)
        iters = 5 if M >= 4224 else 20
        t_gu = timeit(lambda: ops.wq_gemm(ops.W4A8, gq, gs, xq, xscale=xs, out=gu), iters=iters)
        t_dn = timeit(lambda: ops.wq_gemm(ops.W4A8, dq, ds, aq, xscale=as_, out=out), iters=iters)

        def layer():
            ops.wq_gemm(ops.W4A8, gq, gs, xq, xscale=xs, out=gu)
            a8, a8s = ops.silu_mul(gu, quant=True)
            ops.wq_gemm(ops.W4A8, dq, ds, a8, xscale=a8s, out=out)
        t_l = timeit(layer, iters=iters)
        wbytes = gq.numel() * 4 + gs.numel() * 2 + dq.numel() * 4 + ds.numel() * 2
        report("w4a8 mlp gate_up M=%d" % M, t_gu, flops=2 * M * 2 * I * H)
        report("w4a8 mlp down M=%d" % M, t_dn, flops=2 * M * H * I)
        report("w4a8 mlp layer M=%d" % M, t_l, bytes_=wbytes, flops=2 * M * 3 * I * H)


def fill_cache(ctx, nseq, hkv, gqa):
    layout = b200_layout(hkv, gqa)
    pages_per = (ctx + 15) // 16
    pages = pages_per * nseq
    cache = torch.empty(pages, layout.page_bytes, dtype=torch.uint8, device="cuda")
    chunk = 8192
    for s in range(nseq):
        for t0 in range(0, ctx, chunk):
            n = min(chunk, ctx - t0)
            k = torch.randn(n, hkv, 128, device="cuda").bfloat16()
            v = torch.randn(n, hkv, 128, device="cuda").bfloat16()
            slots = torch.arange(t0, t0 + n, device="cuda") + s * pages_per * 16
            ops.kv_store(k, v, slots, cache, hkv)
    bt = (torch.arange(pages, dtype=torch.int32, device="cuda").view(nseq, pages_per))
    return layout, cache, bt


def bench_attn(ctx):
    hkv, gqa = 4, 6
    for nseq in (1, 4):
        layout, cache, bt = fill_cache(ctx, nseq, hkv, gqa)
        lens = torch.full((nseq,), ctx, dtype=torch.int32, device="cuda")
        kv_bytes = nseq * ctx * hkv * 202
        for q_len in (1, 7):
            q = torch.randn(nseq * q_len, hkv * gqa, 128, device="cuda").bfloat16()
            cu = torch.arange(0, nseq * q_len + 1, q_len, dtype=torch.int32, device="cuda")
            for nsplit in (16, 37, 64):
                ws = torch.empty(ops.decode_ws_floats(nseq, hkv, nsplit, q_len, gqa), device="cuda")
                t = timeit(lambda: ops.decode_attn(q, cu, lens, bt, cache, hkv, gqa, q_len, nsplit=nsplit, ws=ws))
                report("decode_attn ctx=%d c=%d q=%d split=%d" % (ctx, nseq, q_len, nsplit), t, bytes_=kv_bytes)
        del cache
    # prefill: one 4224-token chunk at the end of the context
    layout, cache, bt = fill_cache(ctx, 1, hkv, gqa)
    ql = 4224
    q = torch.randn(ql, hkv * gqa, 128, device="cuda").bfloat16()
    cu = torch.tensor([0, ql], dtype=torch.int32, device="cuda")
    lens = torch.tensor([ctx], dtype=torch.int32, device="cuda")
    t = timeit(lambda: ops.prefill_attn(q, cu, lens, bt, cache, hkv, gqa, ql), iters=5, warmup=2)
    keys = ctx - ql + ql / 2
    flops = 4 * hkv * gqa * 128 * ql * keys
    report("prefill_attn q=%d ctx=%d" % (ql, ctx), t, flops=flops)


def bench_attn_libraries(ctx):
    """The reference's flash-vs-oneDNN comparison (``bench/prefill_flash_paged.py``)
    on B200: this framework's paged K8/V4 prefill attention against library
    attention (flash_attn's varlen kernel and torch SDPA) given the same K/V
    dequantized to dense bf16, one 4,224-token chunk at the end of ``ctx``
    keys. The libraries read 2 x 128 x 2 bytes per key and head instead of
    202; each row reports its max difference from ours."""
    hkv, gqa, ql = 4, 6, 4224
    layout, cache, bt = fill_cache(ctx, 1, hkv, gqa)
    q = torch.randn(ql, hkv * gqa, 128, device="cuda").bfloat16()
    cu = torch.tensor([0, ql], dtype=torch.int32, device="cuda")
    lens = torch.tensor([ctx], dtype=torch.int32, device="cuda")
    ours = ops.prefill_attn(q, cu, lens, bt, cache, hkv, gqa, ql)
    t = timeit(lambda: ops.prefill_attn(q, cu, lens, bt, cache, hkv, gqa, ql), iters=5, warmup=2)
    keys = ctx - ql + ql / 2
    flops = 4 * hkv * gqa * 128 * ql * keys
    report("prefill_attn (K8/V4 pages) q=%d ctx=%d" % (ql, ctx), t, flops=flops)
    kd = torch.empty(ctx, hkv, 128, dtype=torch.bfloat16, device="cuda")
    vd = torch.empty_like(kd)
    for h in range(hkv):
        k, v = ops.gather_dequant(cache, bt[0], hkv, h, ctx, dtype=torch.bfloat16)
        kd[:, h], vd[:, h] = k, v
    del cache
    try:
        from flash_attn import flash_attn_varlen_func
        cuq = torch.tensor([0, ql], dtype=torch.int32, device="cuda")
        cuk = torch.tensor([0, ctx], dtype=torch.int32, device="cuda")
        fa = lambda: flash_attn_varlen_func(q, kd, vd, cuq, cuk, ql, ctx, causal=True)  # noqa: E731
        out = fa()
        t = timeit(fa, iters=5, warmup=2)
        report("flash_attn varlen (dense bf16 K/V) q=%d ctx=%d" % (ql, ctx), t, flops=flops,
               max_diff_vs_ours=round((out.float() - ours.float()).abs().max().item(), 4))
    except Exception as e:  # not installed, or no kernel for this GPU
        print(json.dumps({"kernel": "flash_attn varlen", "unavailable": str(e)[:200]}), flush=True)
    try:
        import torch.nn.functional as F
        qh = q.transpose(0, 1).unsqueeze(0)
        kh, vh = kd.transpose(0, 1).unsqueeze(0), vd.transpose(0, 1).unsqueeze(0)
        # bottom-right causal: query i sees keys [0, ctx - ql + i]
        mask = torch.ones(ql, ctx, dtype=torch.bool, device="cuda").tril(ctx - ql)
        sd = lambda: F.scaled_dot_product_attention(qh, kh, vh, attn_mask=mask, enable_gqa=True)  # noqa: E731
        out = sd().squeeze(0).transpose(0, 1)
        t = timeit(sd, iters=3, warmup=1)
        report("torch SDPA (dense bf16 K/V, mask) q=%d ctx=%d" % (ql, ctx), t, flops=flops,
               max_diff_vs_ours=round((out.float() - ours.float()).abs().max().item(), 4))
    except Exception as e:
        print(json.dumps({"kernel": "torch SDPA", "unavailable": str(e)[:200]}), flush=True)


def bench_misc():
    H, I = 5120, 17408
    for T in (1, 4224):
        x = torch.randn(T, H, device="cuda").bfloat16()
        r = torch.randn(T, H, device="cuda").bfloat16()
        w = torch.ones(H, device="cuda").bfloat16()
        t = timeit(lambda: ops.rmsnorm(x, w, residual=r))
        report("rmsnorm+res T=%d" % T, t, bytes_=T * H * 2 * 4)
        gu = torch.randn(T, 2 * I, device="cuda").bfloat16()
        t = timeit(lambda: ops.silu_mul(gu))
        report("silu_mul T=%d" % T, t, bytes_=T * I * 2 * 3)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--only", default=None)
    ap.add_argument("--ctx", type=int, default=128197)
    a = ap.parse_args()
    ops.require()
    print(json.dumps({"peaks": {"hbm_gbs": HBM, "bf16_tflops": TF, "source": SRC}}))
    if a.only in (None, "gemm"):
        bench_gemm()
    if a.only in (None, "mlp"):
        bench_mlp()
    if a.only in (None, "attn"):
        bench_attn(a.ctx)
    if a.only in (None, "misc"):
        bench_misc()
    if a.only == "attnlib":  # only on request: the libraries need dense K/V (and SDPA a dense mask)
        bench_attn_libraries(a.ctx)
    assert ops.status() == 0


if __name__ == "__main__":
    main()
