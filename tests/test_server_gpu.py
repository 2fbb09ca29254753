"""The HTTP server over the real engine (tiny decoder, GPU)."""
import json

import pytest
from fastapi.testclient import TestClient

from k8v4_xpu_b200.api.driver import EngineDriver
from k8v4_xpu_b200.api.metrics import ServingMetrics
from k8v4_xpu_b200.api.server import build_app
from k8v4_xpu_b200.api.tokenizer import ByteTokenizer
from k8v4_xpu_b200.models.config import TINY
from k8v4_xpu_b200.runtime.engine import EngineConfig, LLMEngine
from k8v4_xpu_b200.runtime.scheduler import SamplingParams

pytestmark = pytest.mark.gpu


def _cfg(**kw):
    d = dict(model="tiny", max_model_len=1024, max_num_seqs=2, max_num_batched_tokens=64, num_kv_blocks=128,
             device="cuda")
    d.update(kw)
    return EngineConfig(**d)


@pytest.mark.parametrize("spec", [0, 6])
def test_server_streams_engine_tokens(spec):
    prompt = list(range(7, 120))
    ref = LLMEngine(_cfg(speculative_tokens=spec), TINY).generate([prompt], SamplingParams(max_tokens=12,
                                                                                            ignore_eos=True))[0]
    eng = LLMEngine(_cfg(speculative_tokens=spec), TINY)
    metrics = ServingMetrics("tiny")
    driver = EngineDriver(eng, metrics=metrics).start()
    app = build_app(driver, ByteTokenizer(TINY.vocab), "tiny", 1024, metrics)
    with TestClient(app) as c:
        r = c.post("/v1/completions", json={"prompt": prompt, "max_tokens": 12, "ignore_eos": True}).json()
        assert r["choices"][0]["token_ids"] == ref
        with c.stream("POST", "/v1/completions", json={"prompt": prompt, "max_tokens": 12, "ignore_eos": True,
                                                       "stream": True,
                                                       "stream_options": {"include_usage": True}}) as s:
            chunks = [json.loads(ln[6:]) for ln in s.iter_lines() if ln.startswith("data: {")]
        toks = [t for ch in chunks for choice in ch["choices"] for t in choice.get("token_ids", [])]
        assert toks == ref
        assert chunks[-1]["usage"]["completion_tokens"] == 12
        body = c.get("/metrics").text
        assert "vllm:generation_tokens_total" in body
        if spec:
            assert "vllm:spec_decode_num_drafts_total" in body
    driver.stop()
    assert driver.error is None
