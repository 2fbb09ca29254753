"""Probe clients (reference ``profile_request.py`` and ``mtp_probe_client.py``).

``cold``: one cold held-context request, its timings and metrics deltas
(with ``K8V4_PROFILE`` / ``K8V4_ATTN_TIME`` set on the server, the stage and
attention files land beside it). ``mtp``: coding and agent prompts that
exercise speculative decoding; with ``MTP_TOPK_LOG=1`` on the server the
draft top-k log records them.

    python bench/clients/probe.py cold --base URL --tokens 128197
    python bench/clients/probe.py mtp --base URL
"""
from __future__ import annotations

import argparse
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
from common import metric_delta, random_prompt, scrape, stream_completion, write_jsonl  # noqa: E402

MTP_PROMPTS = [
    [{"role": "user", "content": "Implement binary search in Python with tests."}],
    [{"role": "system", "content": "You are an agent with a shell tool."},
     {"role": "user", "content": "List the files in the repo, then summarize the README."}],
]


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("mode", choices=("cold", "mtp"))
    ap.add_argument("--base", default="http://127.0.0.1:8000")
    ap.add_argument("--tokens", type=int, default=128197)
    ap.add_argument("--max-tokens", type=int, default=128)
    ap.add_argument("--vocab", type=int, default=151936)
    ap.add_argument("--out")
    ap.add_argument("--dry-run", action="store_true")
    a = ap.parse_args(argv)
    if a.dry_run:
        write_jsonl(a.out, {"probe": a.mode, "tokens": a.tokens if a.mode == "cold" else None})
        return 0
    before = scrape(a.base)
    if a.mode == "cold":
        r = stream_completion(a.base, random_prompt(a.tokens, a.vocab, seed=1234), a.max_tokens)
        rec = {"probe": "cold", "prompt_tokens": a.tokens,
               **{k: r[k] for k in ("ttft_s", "e2e_s", "n_tokens", "decode_tok_s")}}
    else:
        rs = [stream_completion(a.base, p, a.max_tokens, ignore_eos=False, chat=True) for p in MTP_PROMPTS]
        rec = {"probe": "mtp", "requests": len(rs), "tokens": sum(r["n_tokens"] for r in rs)}
    after = scrape(a.base)
    rec["metrics_delta"] = metric_delta(before, after)
    write_jsonl(a.out, rec)
    return 0


if __name__ == "__main__":
    sys.exit(main())
