"""Prometheus metrics under the ``vllm:`` names the reference's clients scrape.

``bench/serve_coding.py:27-45`` and ``bench/held_curve.py`` of the reference
read vLLM's ``/metrics``; the names here are the same so those clients work
unchanged: request gauges, token counters, TTFT / e2e latency histograms,
KV-cache usage, prefix-cache queries and hits, preemptions, per-request
prefill / decode time, cached and computed prompt tokens, and the
speculative-decoding counters (drafts, draft tokens, accepted tokens,
accepted tokens per position).
"""
from __future__ import annotations

from prometheus_client import CollectorRegistry, Counter, Gauge, Histogram, generate_latest

_LAT = (0.001, 0.005, 0.01, 0.02, 0.04, 0.06, 0.08, 0.1, 0.25, 0.5, 0.75, 1.0, 2.5, 5.0, 7.5, 10.0, 20.0, 40.0,
        80.0, 160.0, 320.0, 640.0)


class ServingMetrics:
    def __init__(self, model_name: str):
        self.registry = CollectorRegistry()
        L = ["model_name"]
        r = self.registry
        self.model = model_name
        self.running = Gauge("vllm:num_requests_running", "Requests in the running batch", L, registry=r)
        self.waiting = Gauge("vllm:num_requests_waiting", "Requests waiting to be scheduled", L, registry=r)
        self.kv_usage = Gauge("vllm:kv_cache_usage_perc", "KV-cache block usage (1 = full)", L, registry=r)
        self.gpu_cache = Gauge("vllm:gpu_cache_usage_perc", "KV-cache block usage (1 = full)", L, registry=r)
        self.prompt_tokens = Counter("vllm:prompt_tokens", "Prefill tokens processed", L, registry=r)
        self.generation_tokens = Counter("vllm:generation_tokens", "Generated tokens", L, registry=r)
        self.requests_success = Counter("vllm:request_success", "Finished requests", L + ["finished_reason"],
                                        registry=r)
        self.preemptions = Counter("vllm:num_preemptions", "Preemptions", L, registry=r)
        self.prefix_queries = Counter("vllm:prefix_cache_queries", "Prompt tokens looked up", L, registry=r)
        self.prefix_hits = Counter("vllm:prefix_cache_hits", "Prompt tokens served from cache", L, registry=r)
        self.ttft = Histogram("vllm:time_to_first_token_seconds", "Time to first token", L, buckets=_LAT,
                              registry=r)
        self.e2e = Histogram("vllm:e2e_request_latency_seconds", "End-to-end request latency", L, buckets=_LAT,
                             registry=r)
        self.tpot = Histogram("vllm:time_per_output_token_seconds", "Inter-token latency", L, buckets=_LAT,
                              registry=r)
        self.iter_tokens = Histogram("vllm:iteration_tokens_total", "Tokens per engine step", L,
                                     buckets=(1, 8, 16, 32, 64, 128, 256, 512, 1024, 2048, 4096, 8192),
                                     registry=r)
        # per finished request (the reference's clients read these:
        # bench/held_curve.py:36-47, bench/serve_coding.py:32-45)
        self.prefill_time = Histogram("vllm:request_prefill_time_seconds", "Admission to first token", L,
                                      buckets=_LAT, registry=r)
        self.decode_time = Histogram("vllm:request_decode_time_seconds", "First token to finish", L,
                                     buckets=_LAT, registry=r)
        self.prompt_cached = Counter("vllm:prompt_tokens_cached", "Prompt tokens served from the prefix cache",
                                     L, registry=r)
        self.kv_computed = Histogram("vllm:request_prefill_kv_computed_tokens", "Prompt tokens computed (not cached)",
                                     L, buckets=(16, 256, 1024, 4096, 16384, 65536, 262144), registry=r)
        self.spec_drafts = Counter("vllm:spec_decode_num_drafts", "Speculative steps x sequences", L, registry=r)
        self.spec_draft_tokens = Counter("vllm:spec_decode_num_draft_tokens", "Draft tokens proposed", L,
                                         registry=r)
        self.spec_accepted = Counter("vllm:spec_decode_num_accepted_tokens", "Draft tokens accepted", L,
                                     registry=r)
        self.spec_accepted_pos = Counter("vllm:spec_decode_num_accepted_tokens_per_pos",
                                         "Accepted draft tokens by position", L + ["position"], registry=r)
        self._last = {}

    def _delta(self, key: str, value: float) -> float:
        d = value - self._last.get(key, 0)
        self._last[key] = value
        return max(0.0, d)

    def observe_engine(self, engine) -> None:
        """Refresh gauges and counters from the engine's own accounting."""
        m = self.model
        sch = engine.scheduler
        self.running.labels(m).set(len(sch.running))
        self.waiting.labels(m).set(len(sch.waiting))
        u = engine.blocks.usage()
        self.kv_usage.labels(m).set(u)
        self.gpu_cache.labels(m).set(u)
        st = engine.stats
        self.prompt_tokens.labels(m).inc(self._delta("prompt", st["prompt_tokens"]))
        self.generation_tokens.labels(m).inc(self._delta("gen", st["generated_tokens"]))
        self.preemptions.labels(m).inc(self._delta("preempt", sch.num_preemptions))
        self.prefix_queries.labels(m).inc(self._delta("pq", engine.blocks.prefix_queries))
        self.prefix_hits.labels(m).inc(self._delta("ph", engine.blocks.prefix_hits))
        its = st.get("iteration_tokens")
        if its:  # drained here (same thread as the engine), so the list stays short
            for t in its:
                self.iter_tokens.labels(m).observe(t)
            its.clear()
        mtp = getattr(engine, "mtp", None)
        if mtp is not None:
            s = mtp.stats
            self.spec_drafts.labels(m).inc(self._delta("sd", s.num_drafts))
            self.spec_draft_tokens.labels(m).inc(self._delta("sdt", s.num_draft_tokens))
            self.spec_accepted.labels(m).inc(self._delta("sa", s.num_accepted_tokens))
            for i, v in enumerate(s.accepted_per_pos):
                self.spec_accepted_pos.labels(m, str(i)).inc(self._delta("sap%d" % i, v))

    def observe_finished(self, seq) -> None:
        m = self.model
        self.requests_success.labels(m, seq.finish_reason or "stop").inc()
        if seq.first_token_time is not None:
            self.ttft.labels(m).observe(max(0.0, seq.first_token_time - seq.arrival))
            if seq.finish_time is not None and len(seq.output) > 1:
                self.tpot.labels(m).observe(
                    max(0.0, (seq.finish_time - seq.first_token_time) / (len(seq.output) - 1)))
        if seq.finish_time is not None:
            self.e2e.labels(m).observe(max(0.0, seq.finish_time - seq.arrival))
        start = getattr(seq, "prefill_start", None)
        if start is not None and seq.first_token_time is not None:
            self.prefill_time.labels(m).observe(max(0.0, seq.first_token_time - start))
            if seq.finish_time is not None:
                self.decode_time.labels(m).observe(max(0.0, seq.finish_time - seq.first_token_time))
        cached = int(getattr(seq, "cached_tokens", 0) or 0)
        self.prompt_cached.labels(m).inc(cached)
        self.kv_computed.labels(m).observe(max(0, len(seq.prompt) - cached))

    def render(self) -> bytes:
        return generate_latest(self.registry)
