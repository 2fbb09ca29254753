"""Capacity validation (reference ``bench/validate_capacity.py``): several long
held histories at once plus one request near the context limit; asserts the
server preempted nothing (``vllm:num_preemptions_total`` unchanged).

    python bench/clients/validate_capacity.py --base URL [--histories 4 --history-tokens 130000 --long 261000]
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
from common import metric_delta, random_prompt, scrape, stream_completion, write_jsonl  # noqa: E402


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--base", default="http://127.0.0.1:8000")
    ap.add_argument("--histories", type=int, default=4)
    ap.add_argument("--history-tokens", type=int, default=130000)
    ap.add_argument("--long", type=int, default=261000)
    ap.add_argument("--max-tokens", type=int, default=32)
    ap.add_argument("--vocab", type=int, default=151936)
    ap.add_argument("--out")
    ap.add_argument("--dry-run", action="store_true")
    a = ap.parse_args(argv)
    lens = [a.history_tokens] * a.histories + [a.long]
    if a.dry_run:
        write_jsonl(a.out, {"bench": "validate_capacity", "requests": lens})
        return 0
    before = scrape(a.base)
    with cf.ThreadPoolExecutor(len(lens)) as ex:
        rs = list(ex.map(lambda i: stream_completion(a.base, random_prompt(lens[i], a.vocab, seed=7 + i),
                                                     a.max_tokens), range(len(lens))))
    after = scrape(a.base)
    d = metric_delta(before, after, ["vllm:num_preemptions_total"])
    ok = d["vllm:num_preemptions_total"] == 0 and all(r["n_tokens"] == a.max_tokens for r in rs)
    write_jsonl(a.out, {"bench": "validate_capacity", "requests": lens, "preemptions": d[
        "vllm:num_preemptions_total"], "ok": ok})
    return 0 if ok else 1


if __name__ == "__main__":
    sys.exit(main())
