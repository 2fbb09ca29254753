#!/usr/bin/env python3
"""Decode-attention sweep under CUDA-graph replay (reference ``bench/graph_sweep.py``).

Synthetic K8/V4 cache at a held context; for each split count and query
width, captures one decode_attn launch in a CUDA graph, replays it
(CUDA events, L2 flushed between replays) and checks it against the
one-split result of the same inputs.

    python bench/graph_sweep.py [--ctx 128197] [--nseq 1] [--splits 8 16 37 64] [--q 1 7]
"""
from __future__ import annotations

import argparse
import json
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "bench"))

import torch  # noqa: E402

from k8v4_xpu_b200 import ops  # noqa: E402
from microbench import HBM, fill_cache, timeit  # noqa: E402


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--ctx", type=int, default=128197)
    ap.add_argument("--nseq", type=int, default=1)
    ap.add_argument("--splits", type=int, nargs="+", default=[8, 16, 37, 64])
    ap.add_argument("--q", type=int, nargs="+", default=[1, 7])
    a = ap.parse_args(argv)
    ops.require()
    hkv, gqa = 4, 6
    _, cache, bt = fill_cache(a.ctx, a.nseq, hkv, gqa)
    lens = torch.full((a.nseq,), a.ctx, dtype=torch.int32, device="cuda")
    kv_bytes = a.nseq * a.ctx * hkv * 202
    for q_len in a.q:
        q = torch.randn(a.nseq * q_len, hkv * gqa, 128, device="cuda").bfloat16()
        cu = torch.arange(0, a.nseq * q_len + 1, q_len, dtype=torch.int32, device="cuda")
        ref = ops.decode_attn(q, cu, lens, bt, cache, hkv, gqa, q_len, nsplit=1)
        for ns in a.splits:
            ws = torch.empty(ops.decode_ws_floats(a.nseq, hkv, ns, q_len, gqa), dtype=torch.float32, device="cuda")
            out = torch.empty_like(q)
            fn = lambda: ops.decode_attn(q, cu, lens, bt, cache, hkv, gqa, q_len, nsplit=ns, out=out, ws=ws)  # noqa
            us = timeit(fn)
            err = (out.float() - ref.float()).abs().max().item()
            print(json.dumps({"bench": "graph_sweep", "ctx": a.ctx, "nseq": a.nseq, "q_len": q_len, "nsplit": ns,
                              "us": round(us, 2), "hbm_frac": round(kv_bytes / (us * 1e-6) / (HBM * 1e9), 3),
                              "max_err_vs_1split": err, "ok": err < 2e-2}), flush=True)
    st = ops.status()
    print(json.dumps({"status": st}))
    return 0 if st == 0 else 1


if __name__ == "__main__":
    sys.exit(main())
