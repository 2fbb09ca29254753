"""Held-context curve (reference ``bench/held_curve.py``): one request per
context length, ``ignore_eos``, fixed output length; TTFT, prefill tok/s
(prompt / TTFT), decode tok/s after the first update, /metrics deltas.

    python bench/clients/held_curve.py --base http://127.0.0.1:8000 --lengths 2184 8190 128197 [--dry-run]
"""
from __future__ import annotations

import argparse
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
from common import metric_delta, random_prompt, scrape, stream_completion, write_jsonl  # noqa: E402


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--base", default="http://127.0.0.1:8000")
    ap.add_argument("--lengths", type=int, nargs="+", default=[2184, 8190, 128197, 200191])
    ap.add_argument("--max-tokens", type=int, default=96)
    ap.add_argument("--vocab", type=int, default=151936)
    ap.add_argument("--out")
    ap.add_argument("--dry-run", action="store_true")
    a = ap.parse_args(argv)
    for i, n in enumerate(a.lengths):
        plan = {"bench": "held_curve", "prompt_tokens": n, "max_tokens": a.max_tokens, "ignore_eos": True}
        if a.dry_run:
            write_jsonl(a.out, plan)
            continue
        before = scrape(a.base)
        r = stream_completion(a.base, random_prompt(n, a.vocab, seed=i), a.max_tokens)
        after = scrape(a.base)
        plan.update({k: r[k] for k in ("ttft_s", "e2e_s", "n_tokens", "decode_tok_s", "finish_reason")})
        plan["prefill_tok_s"] = n / r["ttft_s"] if r["ttft_s"] else None
        plan["metrics_delta"] = metric_delta(before, after, ["vllm:prompt_tokens_total",
                                                             "vllm:generation_tokens_total",
                                                             "vllm:prefix_cache_hits_total",
                                                             "vllm:num_preemptions_total"])
        write_jsonl(a.out, plan)
    return 0


if __name__ == "__main__":
    sys.exit(main())
