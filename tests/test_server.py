"""OpenAI-compatible server against a CPU engine stand-in (CPU)."""
import json
import time

import pytest
from fastapi.testclient import TestClient

from fakes import FakeEngine
from k8v4_xpu_b200.api.driver import EngineDriver
from k8v4_xpu_b200.api.metrics import ServingMetrics
from k8v4_xpu_b200.api.server import build_app
from k8v4_xpu_b200.api.tokenizer import ByteTokenizer


@pytest.fixture
def client():
    eng = FakeEngine(max_model_len=512)
    metrics = ServingMetrics("tiny")
    driver = EngineDriver(eng, metrics=metrics).start()
    app = build_app(driver, ByteTokenizer(1000), "tiny", 512, metrics)
    with TestClient(app) as c:
        yield c, eng, driver
    driver.stop()


def test_health_models_metrics(client):
    c, eng, driver = client
    assert c.get("/health").json() == {"status": "ok"}
    m = c.get("/v1/models").json()
    assert m["data"][0]["id"] == "tiny" and m["data"][0]["max_model_len"] == 512
    r = c.post("/v1/completions", json={"prompt": [5, 6, 7], "max_tokens": 4, "ignore_eos": True})
    assert r.status_code == 200
    body = c.get("/metrics").text
    for name in ("vllm:prompt_tokens_total", "vllm:generation_tokens_total", "vllm:num_requests_running",
                 "vllm:kv_cache_usage_perc", "vllm:time_to_first_token_seconds_bucket",
                 "vllm:e2e_request_latency_seconds_count", "vllm:prefix_cache_queries_total",
                 "vllm:request_prefill_time_seconds_sum", "vllm:request_decode_time_seconds_count",
                 "vllm:prompt_tokens_cached_total", "vllm:request_prefill_kv_computed_tokens_sum"):
        assert name in body, name
    assert 'vllm:generation_tokens_total{model_name="tiny"} 4.0' in body
    assert 'vllm:request_prefill_kv_computed_tokens_sum{model_name="tiny"} 3.0' in body


def test_completion_tokens_and_usage(client):
    c, *_ = client
    r = c.post("/v1/completions", json={"prompt": [10, 11], "max_tokens": 5, "ignore_eos": True}).json()
    assert r["choices"][0]["token_ids"] == [12, 13, 14, 15, 16]
    assert r["choices"][0]["finish_reason"] == "length"
    assert r["usage"] == {"prompt_tokens": 2, "completion_tokens": 5, "total_tokens": 7}
    # text prompts go through the byte tokenizer
    r = c.post("/v1/completions", json={"prompt": "ab", "max_tokens": 2, "ignore_eos": True}).json()
    assert r["usage"]["prompt_tokens"] == 2
    # stop tokens end the request early
    r = c.post("/v1/completions", json={"prompt": [10], "max_tokens": 9, "stop_token_ids": [13]}).json()
    assert r["choices"][0]["token_ids"] == [11, 12, 13] and r["choices"][0]["finish_reason"] == "stop"


def test_streaming_chat_with_usage(client):
    c, *_ = client
    with c.stream("POST", "/v1/chat/completions",
                  json={"messages": [{"role": "user", "content": "hi"}], "max_tokens": 6, "stream": True,
                        "ignore_eos": True,
                        "stream_options": {"include_usage": True, "continuous_usage_stats": True}}) as r:
        lines = [ln for ln in r.iter_lines() if ln.startswith("data: ")]
    assert lines[-1] == "data: [DONE]"
    chunks = [json.loads(ln[6:]) for ln in lines[:-1]]
    assert chunks[0]["choices"][0]["delta"]["role"] == "assistant"
    toks = [t for ch in chunks for choice in ch["choices"] for t in choice.get("token_ids", [])]
    assert len(toks) == 6
    assert chunks[-1]["choices"] == [] and chunks[-1]["usage"]["completion_tokens"] == 6
    assert all("usage" in ch for ch in chunks)  # continuous usage stats
    fins = [choice["finish_reason"] for ch in chunks for choice in ch["choices"] if choice["finish_reason"]]
    assert fins == ["length"]


def test_concurrent_requests_and_limits(client):
    c, eng, driver = client
    import concurrent.futures as cf
    with cf.ThreadPoolExecutor(4) as ex:
        futs = [ex.submit(c.post, "/v1/completions",
                          json={"prompt": list(range(100 * i, 100 * i + 20)), "max_tokens": 8, "ignore_eos": True})
                for i in range(1, 7)]
        outs = [f.result().json() for f in futs]
    for i, o in enumerate(outs, 1):
        assert o["choices"][0]["token_ids"][0] == 100 * i + 20
    assert c.post("/v1/completions", json={"prompt": [1] * 500, "max_tokens": 20}).status_code == 400
    assert c.post("/v1/completions", json={"prompt": [1], "max_tokens": 2, "n": 17}).status_code == 400
    assert c.post("/v1/completions", json={"prompt": [1], "max_tokens": 2, "n": 0}).status_code == 400
    eng.blocks.check_invariants()
    assert driver.healthy


def test_engine_failure_turns_health_red():
    eng = FakeEngine()

    def boom():
        raise RuntimeError("device status 0x201: mbarrier wait timed out")
    eng.step = boom
    driver = EngineDriver(eng).start()
    app = build_app(driver, ByteTokenizer(1000), "tiny", 512)
    with TestClient(app) as c:
        r = c.post("/v1/completions", json={"prompt": [1, 2], "max_tokens": 2})
        assert r.status_code == 500
        h = c.get("/health")
        assert h.status_code == 503 and "mbarrier" in h.json()["detail"]
        assert c.post("/v1/completions", json={"prompt": [1, 2], "max_tokens": 2}).status_code == 503
    driver.stop()


def test_request_validation_and_non_streaming_chat(client):
    c, eng, _ = client
    bad = [
        {"prompt": [1, 2], "max_tokens": 0},          # max_tokens must be positive
        {"prompt": [], "max_tokens": 2},              # empty prompt
        {"prompt": ["a", "b"], "max_tokens": 2},      # one prompt per request
    ]
    for body in bad:
        assert c.post("/v1/completions", json=body).status_code == 400, body
    assert c.post("/v1/completions", json={"max_tokens": 2}).status_code == 422  # no prompt at all
    r = c.post("/v1/completions", json={"prompt": ["ab"], "max_tokens": 1, "ignore_eos": True}).json()
    assert r["usage"]["prompt_tokens"] == 2 and r["object"] == "text_completion"
    r = c.post("/v1/chat/completions", json={"messages": [{"role": "user", "content": "hi"}], "max_tokens": 3,
                                            "ignore_eos": True}).json()
    msg = r["choices"][0]["message"]
    assert msg["role"] == "assistant" and isinstance(msg["content"], str)
    assert r["usage"]["completion_tokens"] == 3 and r["object"] == "chat.completion"
    eng.blocks.check_invariants()


def test_concurrent_requests_under_kv_pressure_keep_every_token():
    """A pool too small for all requests at once forces recompute preemption
    mid-generation; every response still carries exactly max_tokens tokens
    that follow the fake model's rule (next = last + 1)."""
    import concurrent.futures as cf
    # a short pause per step keeps the requests overlapping even when the
    # host is loaded (the pressure, and so the preemption, needs them at once)
    eng = FakeEngine(max_num_seqs=4, budget=48, num_blocks=10, max_model_len=160, step_delay=0.002)
    driver = EngineDriver(eng).start()
    app = build_app(driver, ByteTokenizer(1000), "tiny", 160)
    with TestClient(app) as c:
        def one(i):
            prompt = list(range(10 * i, 10 * i + 30))
            r = c.post("/v1/completions", json={"prompt": prompt, "max_tokens": 40, "ignore_eos": True})
            return prompt, r.json()
        with cf.ThreadPoolExecutor(6) as ex:
            results = list(ex.map(one, range(1, 9)))
        for prompt, r in results:
            toks = r["choices"][0]["token_ids"]
            assert len(toks) == 40 and r["usage"]["completion_tokens"] == 40
            seq = prompt + toks
            assert all(seq[len(prompt) + j] == (seq[len(prompt) + j - 1] + 1) % 1000 for j in range(40))
    assert eng.scheduler.num_preemptions > 0
    eng.blocks.check_invariants()
    driver.stop()


def test_incremental_decoder_never_splits_a_character():
    import random
    from k8v4_xpu_b200.api.tokenizer import IncrementalDecoder
    tok = ByteTokenizer(1000)
    text = "héllo wörld, 日本語のテキスト 🎉🚀 ok"
    ids = tok.encode(text)
    rng = random.Random(0)
    for _ in range(200):
        dec, out, i = IncrementalDecoder(tok), [], 0
        while i < len(ids):
            n = rng.randrange(0, 4)
            piece = dec.push(ids[i:i + n], final=i + n >= len(ids))
            assert "�" not in piece
            out.append(piece)
            i += n
        out.append(dec.push([], final=True))
        assert "".join(out) == text
    # bytes that never form a character still come out, at the end at the latest
    bad = tok.encode("a") + [0xE6 + 3, 0x97 + 3] + tok.encode("b")
    dec = IncrementalDecoder(tok)
    streamed = "".join(dec.push([t]) for t in bad) + dec.push([], final=True)
    assert streamed == tok.decode(bad)


def test_streamed_text_equals_one_decode_of_the_streamed_tokens(client):
    c, *_ = client
    # ids 0xC3+3, 0xA9+3 ... : the fake model counts up through multi-byte UTF-8 lead/continuation bytes
    texts, ids = [], []
    with c.stream("POST", "/v1/completions", json={"prompt": [0xC2 + 3], "max_tokens": 12, "ignore_eos": True,
                                                   "stream": True}) as r:
        for line in r.iter_lines():
            if not line.startswith("data: ") or line == "data: [DONE]":
                continue
            ch = json.loads(line[6:])["choices"]
            if ch:
                texts.append(ch[0]["text"])
                ids += ch[0]["token_ids"]
    assert len(ids) == 12
    assert "".join(texts) == ByteTokenizer(1000).decode(ids)


def test_a_request_the_engine_refuses_fails_alone():
    """The engine enforces a shorter max_model_len than the HTTP layer knows:
    the refused request gets a 400 (or an error event when streaming) and the
    server keeps serving."""
    eng = FakeEngine(max_model_len=64)
    driver = EngineDriver(eng).start()
    app = build_app(driver, ByteTokenizer(1000), "tiny", 512)
    with TestClient(app) as c:
        r = c.post("/v1/completions", json={"prompt": list(range(3, 103)), "max_tokens": 4})
        assert r.status_code == 400 and "max_model_len" in r.json()["detail"]
        with c.stream("POST", "/v1/completions", json={"prompt": list(range(3, 103)), "max_tokens": 4,
                                                       "stream": True}) as s:
            lines = [ln for ln in s.iter_lines() if ln.startswith("data: ")]
        assert "error" in json.loads(lines[0][6:])
        ok = c.post("/v1/completions", json={"prompt": [10, 11], "max_tokens": 3, "ignore_eos": True})
        assert ok.status_code == 200 and ok.json()["choices"][0]["token_ids"] == [12, 13, 14]
        assert driver.healthy
    driver.stop()


def test_iteration_token_history_is_drained_by_the_exporter(client):
    c, eng, driver = client
    for i in range(3):
        assert c.post("/v1/completions", json={"prompt": [5 + i], "max_tokens": 3, "ignore_eos": True}).status_code == 200
    body = c.get("/metrics").text
    count = [ln for ln in body.splitlines() if ln.startswith("vllm:iteration_tokens_total_count")]
    assert count and float(count[0].split()[-1]) >= 3
    assert len(eng.stats["iteration_tokens"]) <= 1  # drained after each step (one may be in flight)


def test_sampling_fields_reach_the_engine_and_bad_ones_are_refused(client):
    c, eng, driver = client
    seen = []
    orig = eng.add_request

    def spy(prompt, params=None):
        seen.append(params)
        return orig(prompt, params)
    eng.add_request = spy
    r = c.post("/v1/completions", json={"prompt": [1, 2, 3], "max_tokens": 2, "ignore_eos": True,
                                        "temperature": 0.7, "top_p": 0.9, "top_k": -1, "seed": 11})
    assert r.status_code == 200
    p = seen[-1]
    assert (p.temperature, p.top_p, p.top_k, p.seed) == (0.7, 0.9, 0, 11)
    r = c.post("/v1/completions", json={"prompt": [1, 2, 3], "max_tokens": 2, "ignore_eos": True})
    assert r.status_code == 200 and seen[-1].temperature == 0.0  # no temperature: greedy
    for bad in ({"temperature": -0.5}, {"top_p": 0.0}, {"top_p": 1.5}, {"top_k": -3}):
        body = {"prompt": [1, 2], "max_tokens": 2, **bad}
        assert c.post("/v1/completions", json=body).status_code == 400, bad


def test_stop_matcher_holds_back_possible_starts():
    from k8v4_xpu_b200.api.tokenizer import StopMatcher
    m = StopMatcher(["cde", "zz"])
    assert m.feed("ab") == ("", False)        # "ab" might start a stop string: held (2 characters)
    assert m.feed("c") == ("a", False)
    assert m.feed("d") == ("b", False)
    assert m.feed("ef") == ("", True)         # "cde" completes: nothing from it on is shown
    m = StopMatcher(["cde"])
    shown = "".join(m.feed(ch)[0] for ch in "xyzab")
    assert shown == "xyz"
    assert m.feed("cdef") == ("ab", True) and m.feed("more") == ("", True)
    m = StopMatcher(["\n\n"])
    assert m.feed("line\n") == ("line", False) and m.feed("next", final=True) == ("\nnext", False)
    p = StopMatcher(None)
    assert p.feed("abc") == ("abc", False) and p.feed("", final=True) == ("", False)


def test_stop_strings_end_requests_streamed_and_not(client):
    """The stand-in engine continues a prompt byte by byte (next id = last + 1):
    after "a" it writes "bcdefg...". A stop string ends the request before it
    (finish reason "stop") and the engine drops the sequence."""
    c, eng, _ = client
    a = ord("a") + 3  # byte-tokenizer id of "a"
    body = {"prompt": [a], "max_tokens": 20, "ignore_eos": True, "stop": ["ef", "zz"]}
    r = c.post("/v1/completions", json=body).json()
    ch = r["choices"][0]
    assert ch["text"] == "bcd" and ch["finish_reason"] == "stop"
    chunks = []
    with c.stream("POST", "/v1/completions", json={**body, "stream": True}) as s:
        for line in s.iter_lines():
            if line.startswith("data: ") and line != "data: [DONE]":
                chunks.append(json.loads(line[6:]))
    text = "".join(x["choices"][0]["text"] for x in chunks if x["choices"])
    assert text == "bcd" and chunks[-1]["choices"][0]["finish_reason"] == "stop"
    r = c.post("/v1/completions", json={"prompt": [a], "max_tokens": 4, "ignore_eos": True, "stop": "zz"}).json()
    assert r["choices"][0]["text"] == "bcde" and r["choices"][0]["finish_reason"] == "length"
    deadline = time.monotonic() + 5
    while eng.has_unfinished() and time.monotonic() < deadline:
        time.sleep(0.01)
    assert not eng.has_unfinished()  # the stopped requests were dropped, not left decoding
    eng.blocks.check_invariants()


def test_n_choices_streamed_and_not(client):
    """n choices come back with their indices, usage counts every choice's
    tokens once, and a stream interleaves the choices' chunks."""
    c, eng, _ = client
    body = {"prompt": [ord("a") + 3], "max_tokens": 3, "ignore_eos": True, "n": 3}
    r = c.post("/v1/completions", json=body).json()
    assert [ch["index"] for ch in r["choices"]] == [0, 1, 2]
    assert all(ch["text"] == "bcd" and ch["finish_reason"] == "length" for ch in r["choices"])
    assert r["usage"] == {"prompt_tokens": 1, "completion_tokens": 9, "total_tokens": 10}
    texts = {0: "", 1: "", 2: ""}
    fins = {}
    with c.stream("POST", "/v1/chat/completions", json={"messages": [{"role": "user", "content": "x"}],
                                                        "max_tokens": 3, "ignore_eos": True, "n": 3,
                                                        "stream": True}) as s:
        for line in s.iter_lines():
            if line.startswith("data: ") and line != "data: [DONE]":
                ch = json.loads(line[6:])["choices"][0]
                texts[ch["index"]] += ch["delta"].get("content", "")
                if ch["finish_reason"]:
                    fins[ch["index"]] = ch["finish_reason"]
    assert fins == {0: "length", 1: "length", 2: "length"}
    assert len({t for t in texts.values()}) == 1 and texts[0]
    eng.blocks.check_invariants()


def test_logprobs_in_completions_and_chat(client):
    """The stand-in engine reports log-probability -0.5 for each token it
    emits and a made-up top list; the server formats them the OpenAI way."""
    c, eng, _ = client
    a = ord("a") + 3
    r = c.post("/v1/completions", json={"prompt": [a], "max_tokens": 3, "ignore_eos": True, "logprobs": 2}).json()
    lp = r["choices"][0]["logprobs"]
    assert lp["tokens"] == ["b", "c", "d"] and lp["token_logprobs"] == [-0.5, -0.5, -0.5]
    assert lp["top_logprobs"][0] == {"b": -0.5, "c": -1.5} and lp["text_offset"] == [0, 1, 2]
    r = c.post("/v1/completions", json={"prompt": [a], "max_tokens": 2, "ignore_eos": True}).json()
    assert r["choices"][0]["logprobs"] is None  # not asked for
    r = c.post("/v1/chat/completions", json={"messages": [{"role": "user", "content": "x"}], "max_tokens": 2,
                                             "ignore_eos": True, "logprobs": True, "top_logprobs": 1}).json()
    content = r["choices"][0]["logprobs"]["content"]
    assert len(content) == 2 and all(e["logprob"] == -0.5 and len(e["top_logprobs"]) == 1 for e in content)
    assert content[0]["bytes"] == list(content[0]["token"].encode("utf-8"))
    got = []
    with c.stream("POST", "/v1/completions", json={"prompt": [a], "max_tokens": 3, "ignore_eos": True,
                                                   "logprobs": 0, "stream": True}) as s:
        for line in s.iter_lines():
            if line.startswith("data: ") and line != "data: [DONE]":
                ch = json.loads(line[6:])["choices"]
                if ch and ch[0].get("logprobs"):
                    got.append(ch[0]["logprobs"])
    assert [t for g in got for t in g["tokens"]] == ["b", "c", "d"]
    assert [o for g in got for o in g["text_offset"]] == [0, 1, 2]
    assert all(x == {} for g in got for x in g["top_logprobs"])  # logprobs 0: no top list
    for bad in ({"logprobs": 21}, {"logprobs": -1}):
        assert c.post("/v1/completions", json={"prompt": [a], "max_tokens": 2, **bad}).status_code == 400


def test_echo_returns_the_prompt_and_its_logprobs(client):
    c, eng, _ = client
    a = ord("a") + 3
    prompt = [a, a + 1]  # "ab"
    r = c.post("/v1/completions", json={"prompt": prompt, "max_tokens": 2, "ignore_eos": True, "echo": True}).json()
    assert r["choices"][0]["text"] == "abcd" and r["usage"]["completion_tokens"] == 2
    r = c.post("/v1/completions", json={"prompt": prompt, "max_tokens": 1, "ignore_eos": True, "echo": True,
                                        "logprobs": 1}).json()
    lp = r["choices"][0]["logprobs"]
    assert lp["tokens"] == ["a", "b", "c"] and lp["token_logprobs"] == [None, -1.0, -0.5]
    assert lp["text_offset"] == [0, 1, 2]
    chunks = []
    with c.stream("POST", "/v1/completions", json={"prompt": prompt, "max_tokens": 2, "ignore_eos": True,
                                                   "echo": True, "logprobs": 0, "stream": True}) as s:
        for line in s.iter_lines():
            if line.startswith("data: ") and line != "data: [DONE]":
                chunks.append(json.loads(line[6:])["choices"][0])
    assert "".join(ch["text"] for ch in chunks) == "abcd"
    assert [t for ch in chunks if ch.get("logprobs") for t in ch["logprobs"]["token_logprobs"]] == \
        [None, -1.0, -0.5, -0.5]


def test_prompt_scoring_with_echo_and_no_new_tokens(client):
    """``echo`` with ``max_tokens`` 0 (how evaluation harnesses score a
    prompt): the prompt and its log-probabilities, no completion tokens."""
    c, eng, _ = client
    a = ord("a") + 3
    r = c.post("/v1/completions", json={"prompt": [a, a + 1, a + 2], "max_tokens": 0, "echo": True,
                                        "logprobs": 1}).json()
    ch = r["choices"][0]
    assert ch["text"] == "abc" and ch["logprobs"]["token_logprobs"] == [None, -1.0, -1.0]
    assert r["usage"]["completion_tokens"] == 0 and ch["token_ids"] == []
    assert c.post("/v1/completions", json={"prompt": [a], "max_tokens": 0}).status_code == 400
    assert c.post("/v1/completions", json={"prompt": [a], "max_tokens": 0, "echo": True,
                                           "stream": True}).status_code == 400


def test_tokenize_detokenize_ping_version(client):
    c, _, _ = client
    r = c.post("/tokenize", json={"prompt": "ab"}).json()
    assert r["tokens"] == [ord("a") + 3, ord("b") + 3] and r["count"] == 2 and r["max_model_len"] == 512
    r = c.post("/tokenize", json={"messages": [{"role": "user", "content": "hi"}]}).json()
    assert r["count"] > 2
    assert c.post("/tokenize", json={}).status_code == 400
    assert c.post("/detokenize", json={"tokens": [ord("a") + 3, ord("b") + 3]}).json() == {"prompt": "ab"}
    assert c.get("/ping").json() == {"status": "ok"}
    assert c.get("/version").json()["version"]


def test_stop_string_can_be_kept_in_the_output(client):
    from k8v4_xpu_b200.api.tokenizer import StopMatcher
    m = StopMatcher(["cd", "c"], include=True)
    assert m.feed("abcde") == ("abc", True)  # the earliest match ("c" at 2) ends the text, kept
    c, _, _ = client
    body = {"prompt": [ord("a") + 3], "max_tokens": 20, "ignore_eos": True, "stop": ["ef"],
            "include_stop_str_in_output": True}
    r = c.post("/v1/completions", json=body).json()
    assert r["choices"][0]["text"] == "bcdef" and r["choices"][0]["finish_reason"] == "stop"


def test_unsupported_features_are_refused_not_ignored(client):
    c, _, _ = client
    base = {"prompt": [5, 6], "max_tokens": 2}
    for extra in ({"best_of": 17}, {"use_beam_search": True}, {"response_format": {"type": "json_object"}},
                  {"tools": [{"type": "function", "function": {"name": "f"}}]}, {"guided_regex": "a+"},
                  {"guided_choice": []}):
        assert c.post("/v1/completions", json={**base, **extra}).status_code == 400, extra
    ok = {**base, "best_of": 1, "response_format": {"type": "text"}, "tools": [], "user": "x"}
    assert c.post("/v1/completions", json=ok).status_code == 200


def test_best_of_returns_the_most_likely_candidates(client, monkeypatch):
    """best_of candidates are ranked by their tokens' summed log-probability;
    the stand-in engine scores each candidate by its request order."""
    c, eng, _ = client
    orig = eng.add_request
    count = {"n": 0}

    def add(prompt, params=None):
        seq = orig(prompt, params)
        count["n"] += 1
        seq.rank_score = -float(count["n"])   # later candidates are less likely
        return seq
    eng.add_request = add
    orig_step = eng.step

    def step():
        fin = orig_step()
        for s in list(eng.scheduler.running) + fin:
            if s.logprobs and getattr(s, "rank_score", None) is not None:
                s.logprobs[-1] = (s.rank_score, [])
        return fin
    eng.step = step
    r = c.post("/v1/completions", json={"prompt": [5], "max_tokens": 2, "ignore_eos": True, "best_of": 3,
                                        "n": 1}).json()
    assert len(r["choices"]) == 1 and r["choices"][0]["logprobs"] is None
    assert r["usage"]["completion_tokens"] == 6  # every candidate's tokens count
    assert c.post("/v1/completions", json={"prompt": [5], "max_tokens": 2, "best_of": 3,
                                           "stream": True}).status_code == 400


def test_guided_choice_reaches_the_engine_as_token_sequences(client):
    c, eng, _ = client
    seen = []
    orig = eng.add_request

    def spy(prompt, params=None):
        seen.append(params)
        return orig(prompt, params)
    eng.add_request = spy
    r = c.post("/v1/completions", json={"prompt": [5], "max_tokens": 3, "guided_choice": ["yes", "no"]})
    assert r.status_code == 200
    assert seen[-1].allowed_sequences == (tuple(b + 3 for b in b"yes"), tuple(b + 3 for b in b"no"))
