"""HTTP bench clients against a live server on a CPU engine stand-in, charts (CPU)."""
import json
import os
import socket
import subprocess
import sys
import threading
import time

import pytest
import requests

from fakes import FakeEngine
from k8v4_xpu_b200.api.driver import EngineDriver
from k8v4_xpu_b200.api.metrics import ServingMetrics
from k8v4_xpu_b200.api.server import build_app
from k8v4_xpu_b200.api.tokenizer import ByteTokenizer

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CLIENTS = os.path.join(ROOT, "bench", "clients")


@pytest.fixture(scope="module")
def server():
    import uvicorn
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    eng = FakeEngine(max_num_seqs=4, budget=256, num_blocks=2048, max_model_len=8192, vocab=151936)
    metrics = ServingMetrics("fake")
    driver = EngineDriver(eng, metrics=metrics).start()
    app = build_app(driver, ByteTokenizer(151936), "fake", 8192, metrics)
    srv = uvicorn.Server(uvicorn.Config(app, host="127.0.0.1", port=port, log_level="error"))
    th = threading.Thread(target=srv.run, daemon=True)
    th.start()
    base = "http://127.0.0.1:%d" % port
    for _ in range(100):
        try:
            if requests.get(base + "/health", timeout=1).ok:
                break
        except Exception:
            time.sleep(0.1)
    yield base
    srv.should_exit = True
    th.join(5)
    driver.stop()


def _run(script, *args):
    out = subprocess.run([sys.executable, os.path.join(CLIENTS, script), *args], capture_output=True, text=True,
                         timeout=300)
    assert out.returncode == 0, out.stderr
    return [json.loads(ln) for ln in out.stdout.splitlines() if ln.startswith("{")]


def test_held_curve_measures_streams(server):
    recs = _run("held_curve.py", "--base", server, "--lengths", "300", "1000", "--max-tokens", "12")
    assert [r["prompt_tokens"] for r in recs] == [300, 1000]
    for r in recs:
        assert r["n_tokens"] == 12 and r["finish_reason"] == "length"
        assert r["ttft_s"] > 0 and r["decode_tok_s"] > 0
        assert r["metrics_delta"]["vllm:generation_tokens_total"] == 12
        assert r["metrics_delta"]["vllm:prompt_tokens_total"] == r["prompt_tokens"]


def test_agentic_and_capacity_and_probe(server):
    recs = _run("agentic_batch.py", "--base", server, "--requests", "6", "--workers", "3", "--prompt-tokens",
                "50", "400", "--max-tokens", "8")
    assert recs[-1]["summary"] and recs[-1]["generated"] == 48
    recs = _run("validate_capacity.py", "--base", server, "--histories", "3", "--history-tokens", "1000",
                "--long", "3000", "--max-tokens", "4")
    assert recs[-1]["ok"] and recs[-1]["preemptions"] == 0
    recs = _run("probe.py", "cold", "--base", server, "--tokens", "500", "--max-tokens", "5")
    assert recs[0]["n_tokens"] == 5
    recs = _run("serve_coding.py", "--base", server, "--context", "200", "--max-tokens", "6")
    assert all(r["behaviour_ok"] for r in recs)


def test_dry_runs_need_no_server():
    assert _run("held_curve.py", "--dry-run", "--lengths", "2184", "128197")[1]["prompt_tokens"] == 128197
    assert len(_run("agentic_batch.py", "--dry-run")) == 27
    assert _run("validate_capacity.py", "--dry-run")[0]["requests"] == [130000] * 4 + [261000]


def test_svg_chart(tmp_path):
    data = tmp_path / "r.jsonl"
    data.write_text("\n".join(json.dumps({"n": n, "tok_s": t}) for n, t in ((2184, 136.5), (128197, 91.6))))
    out = tmp_path / "c.svg"
    subprocess.run([sys.executable, os.path.join(ROOT, "bench", "charts.py"), str(data), "--x", "n", "--y",
                    "tok_s", "--out", str(out)], check=True, timeout=60)
    svg = out.read_text()
    assert svg.startswith("<svg") and "polyline" in svg and "91.6" in svg
