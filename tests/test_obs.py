"""Stage buckets, exclusive time, attention timer, MTP top-k log and report (CPU)."""
import json

from k8v4_xpu_b200.obs.attn_time import AttnTimer
from k8v4_xpu_b200.obs.stage_profile import bucket_for, bucket_kernel, exclusive_report, stage
from k8v4_xpu_b200.spec import topk_log as T


def test_bucket_taxonomy():
    assert bucket_for("layers.3.gemm_qkv") == "gemm_qkv"
    assert bucket_for("layers.3.o_proj") == "gemm_o"
    assert bucket_for("layers.3.gate_up") == "gemm_gate_up"
    assert bucket_for("layers.3.down") == "gemm_down"
    assert bucket_for("layers.3.attn") == "attention"
    assert bucket_for("layers.3.rope_store") == "kv_store"
    assert bucket_for("layers.3.input_norm") == "norm"
    assert bucket_for("layers.3.act") == "activation"
    assert bucket_for("layers.3.all_reduce") == "collective"
    assert bucket_for("lm_head") == "lm_head" and bucket_for("sampler.argmax") == "sampler"
    assert bucket_for("mtp.eh_proj") == "gemm_mtp" and bucket_for("embed") == "embedding"
    assert bucket_for("something") == "other"
    assert bucket_kernel("void k8v4::attn::decode_attn_kernel<16>(...)") == "attention"
    assert bucket_kernel("ncclDevKernel_AllReduce_Sum_bf16_RING_LL") == "collective"
    assert bucket_kernel("void k8v4::gemm::wq_gemm_kernel<2, 32, 4, 4, 6, 1, 6>") == "lm_head"
    assert bucket_kernel("void k8v4::gemm::wq_gemm_kernel<0, 16, 8, 4, 4, 16, 16>") == "gemm"
    assert bucket_kernel("k8v4::misc::rmsnorm_kernel<4>") == "norm"


def test_exclusive_time_subtracts_children():
    ranges = [("layers.0.attn", 0.0, 10.0), ("layers.0.gemm_qkv", 1.0, 3.0), ("layers.0.down", 12.0, 15.0),
              ("layers.0.all_reduce", 13.0, 14.0)]
    ex = exclusive_report(ranges)
    assert ex["attention"] == 8.0 and ex["gemm_qkv"] == 2.0
    assert ex["gemm_down"] == 2.0 and ex["collective"] == 1.0
    with stage("layers.0.attn"):  # the profiler is off: a no-op
        pass


class _Ev:
    clock = 0.0

    def __init__(self):
        self.t = None
        self.done = True

    def record(self):
        _Ev.clock += 1.5
        self.t = _Ev.clock

    def query(self):
        return self.done

    def elapsed_time(self, other):
        return other.t - self.t


def test_attention_timer_drains_without_sync(tmp_path):
    path = str(tmp_path / "attn_%d.json")
    t = AttnTimer(path=path, rank=3, event_factory=_Ev)
    with t.span("decode"):
        pass
    with t.span("prefill"):
        pass
    t.pending[-1][2].done = False  # the prefill span has not completed yet
    assert t.drain() == 1
    snap = t.snapshot()
    assert snap["total_ms"] == {"decode": 1.5} and snap["pending"] == 1
    t.pending[-1][2].done = True
    t.drain()
    t.publish()
    d = json.load(open(tmp_path / "attn_3.json"))
    assert d["calls"] == {"decode": 1, "prefill": 1} and d["rank"] == 3


def test_topk_labels_and_report(tmp_path, monkeypatch):
    assert T.label_miss(5, [9, 5, 1], [3.0, 2.99, 1.0])["label"] == "rank2"
    assert T.label_miss(5, [9, 5, 1], [3.0, 2.99, 1.0])["near_tie"]
    assert T.label_miss(1, [9, 5, 1], [3.0, 2.0, 1.0])["label"] == "rank3"
    assert T.label_miss(7, [9, 5, 1, 2, 3, 4, 6, 8], [0.0] * 8)["label"] == "outside_top8"
    topk = [[10 + j, 20 + j, 30 + j] + [0] * 5 for j in range(6)]
    vals = [[1.0, 0.5, 0.2] + [0.0] * 5 for _ in range(6)]
    drafts = [10 + j for j in range(6)]
    rec = T.summarize_step(drafts, topk, vals, [10, 11, 22, 0, 0, 0, 0], accepted=2)
    assert rec["accepted"] == 2 and rec["miss"]["pos"] == 2 and rec["miss"]["label"] == "rank2"
    rec_all = T.summarize_step(drafts, topk, vals, drafts + [0], accepted=6)
    assert rec_all["miss"] is None
    monkeypatch.setenv("MTP_TOPK_LOG", "1")
    monkeypatch.setenv("MTP_TOPK_FILE", str(tmp_path / "log.jsonl"))
    lg = T.TopKLogger.from_env()
    for acc, tgt in ((2, [10, 11, 22, 0, 0, 0, 0]), (0, [20, 0, 0, 0, 0, 0, 0]), (1, [10, 31, 0, 0, 0, 0, 0]),
                     (6, drafts + [0])):
        lg.record(0, drafts, topk, vals, tgt, acc)
        lg.end_step()
    lg.close()
    recs = T.load(str(tmp_path / "log.jsonl"))
    rep = T.report(recs)
    assert rep["records"] == 4 and rep["miss_labels"] == {"rank2": 2, "rank3": 1}
    assert rep["tree_drafting"] == "recommend"
    assert abs(rep["mean_accepted_length"] - (1 + 9 / 4)) < 1e-9
    assert rep["acceptance_by_position"][0] == 0.75
    assert T.main([str(tmp_path / "log.jsonl")]) == 0
