"""Stage profiler over a real forward, MTP top-k logging on the engine (GPU)."""
import json

import pytest
import torch

from k8v4_xpu_b200.models.config import TINY
from k8v4_xpu_b200.obs import stage_profile
from k8v4_xpu_b200.runtime.engine import EngineConfig, LLMEngine
from k8v4_xpu_b200.runtime.scheduler import SamplingParams
from k8v4_xpu_b200.spec import topk_log

pytestmark = pytest.mark.gpu


def _cfg(**kw):
    d = dict(model="tiny", max_model_len=1024, max_num_seqs=2, max_num_batched_tokens=64, num_kv_blocks=128,
             device="cuda", cuda_graphs=False)
    d.update(kw)
    return EngineConfig(**d)


def test_stage_profiler_buckets_a_forward(tmp_path):
    eng = LLMEngine(_cfg(), TINY)
    prof = stage_profile.install(str(tmp_path), rank=0)
    try:
        eng.generate([list(range(1, 100))], SamplingParams(max_tokens=3, ignore_eos=True))
        rep = prof.report()
        path = prof.write()
    finally:
        stage_profile.uninstall()
    ex = rep["exclusive_ms"]
    for b in ("gemm_qkv", "gemm_o", "gemm_gate_up", "gemm_down", "attention", "kv_store", "norm", "lm_head",
              "sampler", "embedding"):
        assert ex[b] > 0, b
    assert json.load(open(path))["ranges"] == rep["ranges"]


def test_mtp_topk_logging(tmp_path, monkeypatch):
    monkeypatch.setenv("MTP_TOPK_LOG", "1")
    monkeypatch.setenv("MTP_TOPK_FILE", str(tmp_path / "topk.jsonl"))
    eng = LLMEngine(_cfg(speculative_tokens=6, cuda_graphs=True), TINY)
    assert eng.mtp.topk_log is not None and not eng.mtp.use_graphs
    eng.generate([list(range(1, 90))], SamplingParams(max_tokens=20, ignore_eos=True))
    eng.mtp.topk_log.close()
    recs = topk_log.load(str(tmp_path / "topk.jsonl"))
    assert recs and all(r["k"] == 6 for r in recs)
    rep = topk_log.report(recs)
    assert rep["records"] == len(recs) and rep["tree_drafting"] in ("recommend", "reject")
    torch.cuda.synchronize()
