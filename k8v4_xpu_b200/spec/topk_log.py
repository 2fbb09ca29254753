"""MTP draft top-k logging (measurement only; ``MTP_TOPK_LOG=1``, ``MTP_TOPK_FILE``).

Behaviour of the reference's logger (``k8v4_v030/mtp_topk_log.py:232-346``)
and report (``mtp_topk_report.py:90-206``): for every speculative step and
sequence, the drafter's top-8 at each draft position is compared with the
verifier's argmax. Accepted positions count as hits; the first rejected
position is labelled by where the verifier's token sat in the drafter's
top-8 (``rank2``, ``rank3``, ``rank4_8``, ``outside_top8``) and whether the
drafter's top-1 and that token were a near tie. The report turns these into
acceptance per position and a tree-drafting recommendation: if a large share
of misses are rank-2/3 tokens, a tree of the top candidates would have
accepted them.

Here the hooks are part of the speculator (no source patching): with logging
on, the drafter runs eagerly (TP1) and keeps ``torch.topk(logits, 8)`` per
draft position.
"""
from __future__ import annotations

import collections
import json
import os
import sys

TOPK = 8
LABELS = ("rank2", "rank3", "rank4_8", "outside_top8")


def label_miss(target: int, topk_ids: list[int], topk_vals: list[float], tie_margin: float = 0.05) -> dict:
    """Where the verifier's ``target`` sat in the drafter's top-k at a missed position."""
    if target in topk_ids:
        r = topk_ids.index(target)  # 0 would have been a hit
        label = "rank2" if r == 1 else "rank3" if r == 2 else "rank4_8"
        gap = float(topk_vals[0] - topk_vals[r])
        return {"label": label, "rank": r + 1, "gap": gap, "near_tie": gap <= tie_margin}
    return {"label": "outside_top8", "rank": None, "gap": None, "near_tie": False}


def summarize_step(drafts: list[int], topk_ids: list[list[int]], topk_vals: list[list[float]], targets: list[int],
                   accepted: int, tie_margin: float = 0.05) -> dict:
    """One sequence, one verify step. ``targets[j]`` is the verifier's argmax
    at the position draft ``j`` was proposed for."""
    k = len(drafts)
    rec = {"k": k, "accepted": int(accepted), "miss": None}
    if accepted < k:
        j = int(accepted)
        m = label_miss(int(targets[j]), list(topk_ids[j]), list(topk_vals[j]), tie_margin)
        m["pos"] = j
        m["draft"] = int(drafts[j])
        m["target"] = int(targets[j])
        rec["miss"] = m
    return rec


def swap_counts(records: list[dict]) -> dict:
    """Histogram of miss labels (and near ties) by draft position."""
    out: dict = collections.defaultdict(lambda: collections.Counter())
    for r in records:
        m = r.get("miss")
        if m is None:
            continue
        out[m["pos"]][m["label"]] += 1
        if m.get("near_tie"):
            out[m["pos"]]["near_tie"] += 1
    return {p: dict(c) for p, c in sorted(out.items())}


class TopKLogger:
    def __init__(self, path: str | None = None, tie_margin: float = 0.05):
        self.path = path or os.environ.get("MTP_TOPK_FILE", "mtp_topk.jsonl")
        self.tie_margin = tie_margin
        self.records: list[dict] = []
        self.step = 0
        self._f = open(self.path, "a")

    @classmethod
    def from_env(cls) -> "TopKLogger | None":
        if os.environ.get("MTP_TOPK_LOG", "0") in ("", "0", "false"):
            return None
        return cls()

    def record(self, seq_id: int, drafts, topk_ids, topk_vals, targets, accepted: int) -> dict:
        rec = summarize_step(list(drafts), topk_ids, topk_vals, list(targets), accepted, self.tie_margin)
        rec["seq"] = int(seq_id)
        rec["step"] = self.step
        self.records.append(rec)
        self._f.write(json.dumps(rec) + "\n")
        return rec

    def end_step(self) -> None:
        self.step += 1
        self._f.flush()

    def close(self) -> None:
        self._f.close()


def report(records: list[dict], tree_threshold: float = 0.30) -> dict:
    """Acceptance per position, miss labels, and the tree-drafting verdict."""
    if not records:
        return {"steps": 0}
    k = max(r["k"] for r in records)
    n = len(records)
    hit = [0] * k
    for r in records:
        for j in range(r["accepted"]):
            hit[j] += 1
    labels = collections.Counter(r["miss"]["label"] for r in records if r.get("miss"))
    misses = sum(labels.values())
    near = sum(1 for r in records if r.get("miss") and r["miss"].get("near_tie"))
    recoverable = labels.get("rank2", 0) + labels.get("rank3", 0)
    share = recoverable / misses if misses else 0.0
    return {
        "records": n, "k": k,
        "mean_accepted_length": 1.0 + sum(r["accepted"] for r in records) / n,
        "acceptance_by_position": [h / n for h in hit],
        "miss_labels": dict(labels), "near_ties": near,
        "rank2_3_share_of_misses": share,
        "tree_drafting": "recommend" if share >= tree_threshold else "reject",
        "by_position": swap_counts(records),
    }


def load(path: str) -> list[dict]:
    with open(path) as f:
        return [json.loads(ln) for ln in f if ln.strip()]


def main(argv=None) -> int:
    argv = sys.argv[1:] if argv is None else argv
    if not argv:
        print("usage: python -m k8v4_xpu_b200.spec.topk_log <mtp_topk.jsonl>")
        return 2
    print(json.dumps(report(load(argv[0])), indent=2))
    return 0


if __name__ == "__main__":
    sys.exit(main())
