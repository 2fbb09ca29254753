"""Coding-task client (reference ``bench/serve_coding.py``): chat requests that
end on their own (natural EOS), decode rate after the first update, and a
behaviour check on the answer (non-empty, finished).

    python bench/clients/serve_coding.py --base URL [--context 2153] [--dry-run]
"""
from __future__ import annotations

import argparse
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
from common import metric_delta, scrape, stream_completion, write_jsonl  # noqa: E402

TASKS = [
    "Write a Python function that returns the n-th Fibonacci number iteratively.",
    "Write a C function that reverses a singly linked list in place.",
    "Write a SQL query that returns the three most recent orders per customer.",
]


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--base", default="http://127.0.0.1:8000")
    ap.add_argument("--context", type=int, default=2153, help="filler characters of held context before the task")
    ap.add_argument("--max-tokens", type=int, default=512)
    ap.add_argument("--out")
    ap.add_argument("--dry-run", action="store_true")
    a = ap.parse_args(argv)
    filler = ("# notes\n" * (a.context // 8 + 1))[: a.context]
    for t in TASKS:
        msgs = [{"role": "system", "content": filler}, {"role": "user", "content": t}]
        rec = {"bench": "serve_coding", "task": t, "context_chars": a.context, "max_tokens": a.max_tokens}
        if a.dry_run:
            write_jsonl(a.out, rec)
            continue
        before = scrape(a.base)
        r = stream_completion(a.base, msgs, a.max_tokens, ignore_eos=False, chat=True)
        after = scrape(a.base)
        rec.update({k: r[k] for k in ("ttft_s", "e2e_s", "n_tokens", "decode_tok_s", "finish_reason")})
        rec["behaviour_ok"] = r["n_tokens"] > 0 and r["finish_reason"] in ("stop", "length")
        rec["metrics_delta"] = metric_delta(before, after, ["vllm:generation_tokens_total"])
        write_jsonl(a.out, rec)
    return 0


if __name__ == "__main__":
    sys.exit(main())
