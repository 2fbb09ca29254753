#!/usr/bin/env python3
"""Small, self-terminating cases of single kernels for ncu captures.

Each case holds at most a few hundred MB on the device (inputs just above the
126 MB L2 so DRAM counters mean something) and launches the kernel a handful
of times, so an ``ncu --set full -k <kernel> -c 1..3`` capture ends by itself.

    python bench/profile_case.py --case decode|decode7|gemm_m1|gemm_prefill|w4a8_prefill|prefill|sp_rs|sp_ag
"""
from __future__ import annotations

import argparse
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import torch  # noqa: E402

from k8v4_xpu_b200 import ops  # noqa: E402
from k8v4_xpu_b200.layers.linear import split_for  # noqa: E402

sys.path.insert(0, os.path.join(ROOT, "bench"))
from microbench import fill_cache, rand_int4  # noqa: E402


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--case", required=True)
    ap.add_argument("--reps", type=int, default=3)
    a = ap.parse_args()
    ops.require()
    c = a.case
    if c in ("decode", "decode7"):
        ctx, hkv, gqa = 160000, 4, 6
        q_len = 7 if c == "decode7" else 1
        layout, cache, bt = fill_cache(ctx, 1, hkv, gqa)
        q = torch.randn(q_len, hkv * gqa, 128, device="cuda").bfloat16()
        cu = torch.tensor([0, q_len], dtype=torch.int32, device="cuda")
        lens = torch.tensor([ctx], dtype=torch.int32, device="cuda")
        fn = lambda: ops.decode_attn(q, cu, lens, bt, cache, hkv, gqa, q_len, nsplit=37)  # noqa: E731
    elif c == "prefill":
        ctx, hkv, gqa, ql = 40000, 4, 6, 4224
        layout, cache, bt = fill_cache(ctx, 1, hkv, gqa)
        q = torch.randn(ql, hkv * gqa, 128, device="cuda").bfloat16()
        cu = torch.tensor([0, ql], dtype=torch.int32, device="cuda")
        lens = torch.tensor([ctx], dtype=torch.int32, device="cuda")
        fn = lambda: ops.prefill_attn(q, cu, lens, bt, cache, hkv, gqa, ql)  # noqa: E731
    elif c == "gemm_m1":
        N, K = 34816, 5120  # gate_up: 89 MB of int4 weights
        qw, sc = rand_int4(N, K)
        x = torch.randn(1, K, device="cuda").bfloat16()
        ws = torch.zeros(N, dtype=torch.float32, device="cuda")
        fn = lambda: ops.wq_gemm(ops.W4A16, qw, sc, x, ws=ws, split=split_for(1, N, K))  # noqa: E731
    elif c in ("gemm_prefill", "w4a8_prefill"):
        N, K, M = 34816, 5120, 4224
        qw, sc = rand_int4(N, K)
        if c == "gemm_prefill":
            x = torch.randn(M, K, device="cuda").bfloat16()
            fn = lambda: ops.wq_gemm(ops.W4A16, qw, sc, x)  # noqa: E731
        else:
            xq = torch.randint(-127, 127, (M, K), dtype=torch.int8, device="cuda")
            xs = torch.rand(M, device="cuda") * 0.01
            fn = lambda: ops.wq_gemm(ops.W4A8, qw, sc, xq, xscale=xs)  # noqa: E731
    elif c in ("sp_rs", "sp_ag"):
        # the sequence-parallel prefill GEMMs of a TP2 rank (W4A8, 4,224-row
        # chunk) on one GPU: the other rank's slot and counters are local
        # buffers and the all-gather counters are preset, so the kernel runs
        # its full epilogue / wait code with no second process
        from k8v4_xpu_b200.parallel.seq_parallel import tile_owners
        M, H, I = 4224, 5120, 17408
        tile0 = tile_owners(M, 2)
        if c == "sp_rs":
            N, K = H, I // 2      # down_proj shard
        else:
            N, K = I, H           # gate/up shard
        qw, sc = rand_int4(N, K)
        xq = torch.randint(-127, 127, (M, K), dtype=torch.int8, device="cuda")
        xs = torch.rand(M, device="cuda") * 0.01
        cnt = torch.zeros(16, dtype=torch.int64, device="cuda")
        if c == "sp_rs":
            rows = max(tile0[o + 1] - tile0[o] for o in range(2)) * 128  # the largest owner's share
            slots = [torch.empty(rows * N, dtype=torch.bfloat16, device="cuda") for _ in range(2)]
            fn = lambda: ops.wq_gemm_sp(ops.W4A8, qw, sc, xq, 2, 0, tile0, xscale=xs,  # noqa: E731
                                         rs_dst=[t.data_ptr() for t in slots],
                                         rs_sig=[cnt.data_ptr(), cnt.data_ptr() + 8])
        else:
            cnt.fill_(1 << 40)  # every owner's rows "arrived"
            fn = lambda: ops.wq_gemm_sp(ops.W4A8, qw, sc, xq, 2, 0, tile0, xscale=xs,  # noqa: E731
                                         ag_flag=cnt.data_ptr(), ag_target=[1, 1])
    elif c in ("decode_step", "decode_step4"):
        # two layers of the 27B decoder, 128K context written straight into
        # the KV pool, one eager decode step per call (kernel launch lists)
        from k8v4_xpu_b200.models.config import DENSE_27B
        from k8v4_xpu_b200.models.dense import DenseModel, StepInputs
        from k8v4_xpu_b200.runtime.workspace import Workspace
        from k8v4_xpu_b200.runtime.engine import decode_splits
        nseq = 4 if c == "decode_step4" else 1
        ctx = 128197
        m = DenseModel(DENSE_27B, device="cuda").random_init(seed=0, layers=2)
        layout = m.layout
        caches = []
        for _ in m.layers:
            _, cache, bt = fill_cache(ctx + 64, nseq, layout.hkv, layout.gqa)
            caches.append(cache)
        ws = Workspace("cuda", 64, nseq, bt.shape[1], 2 * DENSE_27B.intermediate, layout.hkv, layout.gqa, 1, 64)
        pages_per = bt.shape[1]
        pos = torch.full((nseq,), ctx, dtype=torch.int64, device="cuda")
        inp = StepInputs(
            input_ids=torch.randint(0, DENSE_27B.vocab, (nseq,), device="cuda"), positions=pos,
            slots=torch.arange(nseq, device="cuda") * pages_per * 16 + ctx,
            cu_q=torch.arange(nseq + 1, dtype=torch.int32, device="cuda"),
            seq_lens=torch.full((nseq,), ctx + 1, dtype=torch.int32, device="cuda"), block_table=bt,
            logit_rows=torch.arange(nseq, device="cuda"), max_q_len=1, is_decode=True,
            nsplit=decode_splits(8200, nseq, layout.hkv))
        fn = lambda: m.greedy(m.forward(inp, caches, ws))  # noqa: E731
    else:
        raise SystemExit("unknown case %s" % c)
    for _ in range(a.reps):
        fn()
    torch.cuda.synchronize()
    st = ops.status()
    if st:
        raise SystemExit("device status 0x%x" % st)
    print("ok", c)


if __name__ == "__main__":
    main()
