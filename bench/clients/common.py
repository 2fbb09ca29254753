"""Shared pieces of the HTTP bench clients: streaming requests, /metrics scraping.

Timing rules of the reference's clients (``bench/serve_coding.py:27-45,
143-145``): time to first token is measured to the first streamed update
that carries tokens; the decode rate excludes that first update (tokens
after it / time after it); server-side counters come from ``/metrics``
deltas around the request.
"""
from __future__ import annotations

import json
import time

import requests


def parse_metrics(text: str) -> dict[str, float]:
    """Prometheus text -> {series: value}, labels dropped (summed per name)."""
    out: dict[str, float] = {}
    for ln in text.splitlines():
        if not ln or ln.startswith("#"):
            continue
        name_labels, _, val = ln.rpartition(" ")
        name = name_labels.split("{", 1)[0]
        try:
            out[name] = out.get(name, 0.0) + float(val)
        except ValueError:
            continue
    return out


def scrape(base: str) -> dict[str, float]:
    return parse_metrics(requests.get(base.rstrip("/") + "/metrics", timeout=30).text)


def metric_delta(before: dict, after: dict, names=None) -> dict:
    keys = names or sorted(set(before) | set(after))
    return {k: after.get(k, 0.0) - before.get(k, 0.0) for k in keys if k.startswith("vllm:")}


def stream_completion(base: str, prompt, max_tokens: int, ignore_eos: bool = True, chat: bool = False,
                      model: str | None = None, timeout: float = 3600.0) -> dict:
    """One streamed request; returns tokens and timings (seconds)."""
    url = base.rstrip("/") + ("/v1/chat/completions" if chat else "/v1/completions")
    body = {"max_tokens": max_tokens, "stream": True, "ignore_eos": ignore_eos,
            "stream_options": {"include_usage": True}}
    if model:
        body["model"] = model
    if chat:
        body["messages"] = prompt if isinstance(prompt, list) and prompt and isinstance(prompt[0], dict) else [
            {"role": "user", "content": prompt}]
    else:
        body["prompt"] = prompt
    t0 = time.perf_counter()
    first = None
    updates = []
    toks: list[int] = []
    usage = None
    finish = None
    text = []
    with requests.post(url, json=body, stream=True, timeout=timeout) as r:
        r.raise_for_status()
        for raw in r.iter_lines():
            if not raw or not raw.startswith(b"data: "):
                continue
            data = raw[6:]
            if data == b"[DONE]":
                break
            ch = json.loads(data)
            if ch.get("usage") and not ch.get("choices"):
                usage = ch["usage"]
                continue
            for c in ch.get("choices", []):
                ids = c.get("token_ids", [])
                piece = c.get("text") if "text" in c else (c.get("delta") or {}).get("content", "")
                if ids or piece:
                    now = time.perf_counter()
                    if first is None:
                        first = now
                    updates.append((now, len(ids)))
                    toks.extend(ids)
                    text.append(piece or "")
                if c.get("finish_reason"):
                    finish = c["finish_reason"]
    t1 = time.perf_counter()
    after_first = sum(n for _, n in updates[1:])
    decode_s = (updates[-1][0] - updates[0][0]) if len(updates) > 1 else 0.0
    return {"ttft_s": (first - t0) if first else None, "e2e_s": t1 - t0, "tokens": toks, "text": "".join(text),
            "n_tokens": len(toks), "usage": usage, "finish_reason": finish, "updates": len(updates),
            "decode_tok_s": (after_first / decode_s) if decode_s > 0 else None}


def write_jsonl(path: str | None, rec: dict) -> None:
    line = json.dumps(rec)
    print(line, flush=True)
    if path:
        with open(path, "a") as f:
            f.write(line + "\n")


def random_prompt(n: int, vocab: int = 151936, seed: int = 0) -> list[int]:
    import random
    rng = random.Random(seed)
    return [rng.randrange(259, vocab) for _ in range(n)]
