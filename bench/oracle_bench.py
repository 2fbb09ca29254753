#!/usr/bin/env python3
"""the K8/V4 paged decode-attention oracle workload.

4 sequences (1,024 / 2,048 / 3,072 / 4,096 tokens), 24 Q / 4 KV heads,
head_dim 128, page 16 with a shuffled page table, q/k/v from N(0, 1) in bf16
(seed 0). Times the CPU oracle (page gather + dequant + fp32 attention, the
reference's oracle restated for this format: ``k8v4_v030/oracle.py:100-163``)
and, on a GPU, the split-K decode kernel on the same pages, and reports both
against unquantized bf16 SDPA.

    python bench/oracle_bench.py [--reps 5]
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import time

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import torch  # noqa: E402

from k8v4_xpu_b200.kv import layout as L  # noqa: E402
from k8v4_xpu_b200.kv import oracle as O  # noqa: E402
from k8v4_xpu_b200.kv.pack import gather_sequence, store_tokens  # noqa: E402


def build():
    lay = L.b200_layout(4, 6)
    seqs = O.oracle_config(seed=0)
    total = sum((k.shape[0] + 15) // 16 for _, k, _ in seqs)
    perm = torch.randperm(total, generator=torch.Generator().manual_seed(0))
    cache = torch.zeros(total, lay.page_bytes, dtype=torch.uint8)
    tables, off = [], 0
    for q, k, v in seqs:
        n = k.shape[0]
        npg = (n + 15) // 16
        pages = perm[off:off + npg]
        off += npg
        slots = (pages.repeat_interleave(16) * 16 + torch.arange(16).repeat(npg))[:n]
        store_tokens(cache, slots, k, v, lay)
        tables.append(pages.tolist())
    return lay, seqs, cache, tables


def cpu_oracle(lay, seqs, cache, tables):
    outs = []
    for (q, k, _), pages in zip(seqs, tables):
        n = k.shape[0]
        kd, vd = gather_sequence(cache, pages, n, lay)
        outs.append(O.attention_ref(q.float(), kd, vd, [n], lay.gqa))
    return torch.cat(outs, 0)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reps", type=int, default=5)
    a = ap.parse_args()
    lay, seqs, cache, tables = build()
    sdpa = torch.cat([O.sdpa_bf16_ref(q, k, v, lay.gqa) for q, k, v in seqs], 0)
    ref = cpu_oracle(lay, seqs, cache, tables)
    t0 = time.perf_counter()
    for _ in range(a.reps):
        cpu_oracle(lay, seqs, cache, tables)
    cpu_s = (time.perf_counter() - t0) / a.reps
    row = {"bench": "oracle config 1 (4 seqs 1024-4096, 24Q/4KV, D128, page 16)",
           "cpu_oracle_ms": round(cpu_s * 1e3, 3), "cpu_threads": torch.get_num_threads(),
           "oracle_vs_bf16_sdpa_max_abs": round((ref - sdpa).abs().max().item(), 5)}
    if torch.cuda.is_available():
        from k8v4_xpu_b200 import ops
        from k8v4_xpu_b200.runtime.engine import decode_splits
        ops.require()
        dev = torch.device("cuda")
        W = max(len(t) for t in tables)
        bt = torch.zeros(len(tables), W, dtype=torch.int32)
        for i, t in enumerate(tables):
            bt[i, :len(t)] = torch.tensor(t, dtype=torch.int32)
        q = torch.cat([s[0] for s in seqs], 0).to(dev)
        cu = torch.arange(len(seqs) + 1, dtype=torch.int32, device=dev)
        lens = torch.tensor([k.shape[0] for _, k, _ in seqs], dtype=torch.int32, device=dev)
        gcache, gbt = cache.to(dev), bt.to(dev)
        nsplit = decode_splits(W, len(seqs), 4)
        fn = lambda: ops.decode_attn(q, cu, lens, gbt, gcache, 4, 6, 1, nsplit=nsplit)  # noqa: E731
        out = fn()
        torch.cuda.synchronize()
        assert ops.status() == 0
        for _ in range(5):
            fn()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        e0.record()
        for _ in range(50):
            fn()
        e1.record()
        torch.cuda.synchronize()
        row.update(gpu_kernel_us=round(e0.elapsed_time(e1) / 50 * 1e3, 2), nsplit=nsplit,
                   gpu_vs_oracle_max_abs=round((out.float().cpu() - ref).abs().max().item(), 5),
                   gpu_vs_bf16_sdpa_max_abs=round((out.float().cpu() - sdpa).abs().max().item(), 5))
    print(json.dumps(row))


if __name__ == "__main__":
    main()
