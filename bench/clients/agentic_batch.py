"""Agentic overlap workload (reference ``bench/serve_agentic_batch.py``): a
fixed list of requests served by a pool of workers, so prefills overlap
other requests' decodes; per-request timings plus the aggregate decode rate.

    python bench/clients/agentic_batch.py --base URL [--requests 27 --workers 4] [--dry-run]
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import sys
import time

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
from common import random_prompt, stream_completion, write_jsonl  # noqa: E402


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--base", default="http://127.0.0.1:8000")
    ap.add_argument("--requests", type=int, default=27)
    ap.add_argument("--workers", type=int, default=4)
    ap.add_argument("--prompt-tokens", type=int, nargs=2, default=[2000, 12000], metavar=("MIN", "MAX"))
    ap.add_argument("--max-tokens", type=int, default=256)
    ap.add_argument("--vocab", type=int, default=151936)
    ap.add_argument("--out")
    ap.add_argument("--dry-run", action="store_true")
    a = ap.parse_args(argv)
    lo, hi = a.prompt_tokens
    lens = [lo + (hi - lo) * i // max(1, a.requests - 1) for i in range(a.requests)]
    if a.dry_run:
        for i, n in enumerate(lens):
            write_jsonl(a.out, {"bench": "agentic_batch", "request": i, "prompt_tokens": n})
        return 0
    t0 = time.perf_counter()

    def one(i):
        r = stream_completion(a.base, random_prompt(lens[i], a.vocab, seed=100 + i), a.max_tokens)
        return i, r

    toks = 0
    with cf.ThreadPoolExecutor(a.workers) as ex:
        for i, r in ex.map(one, range(a.requests)):
            toks += r["n_tokens"]
            write_jsonl(a.out, {"bench": "agentic_batch", "request": i, "prompt_tokens": lens[i],
                                **{k: r[k] for k in ("ttft_s", "e2e_s", "n_tokens", "decode_tok_s")}})
    wall = time.perf_counter() - t0
    write_jsonl(a.out, {"bench": "agentic_batch", "summary": True, "wall_s": wall, "generated": toks,
                        "aggregate_tok_s": toks / wall})
    return 0


if __name__ == "__main__":
    sys.exit(main())
