"""Per-stage device-time profiler of the decoder (opt-in: ``K8V4_PROFILE=1``).

Behaviour of the reference's stage profiler (``k8v4_v030/stage_profile.py``):
named ranges around the model's stages are timed on the device, folded into
a fixed bucket taxonomy (qkv / o / gate_up / down GEMMs, attention, KV store,
norms, activation, collectives, embedding, lm_head, sampling), and reported
as *exclusive* time (a range's children are subtracted from it) in a JSON
file per process under ``K8V4_PROFILE_DIR``. Kernel names from a
torch.profiler trace fold into the same buckets (``bucket_kernel``).

Here the model calls ``stage("layers.3.gemm_qkv")`` around each op; with the
profiler off that is a shared no-op context manager. Ranges record CUDA events
on the current stream and an NVTX range (visible in Nsight timelines); they are
skipped while a CUDA graph is being captured (decode graphs are timed as a
whole by the caller instead).
"""
from __future__ import annotations

import contextlib
import json
import os
import time

BUCKETS = ("gemm_qkv", "gemm_o", "gemm_gate_up", "gemm_down", "gemm_mtp", "attention", "kv_store", "norm",
           "activation", "collective", "embedding", "lm_head", "sampler", "other")

COLLECTIVE_NAMES = ("all_reduce", "all_gather", "reduce_scatter", "broadcast", "allreduce", "allgather",
                    "reducescatter", "nccl")

_RULES = (
    ("gemm_qkv", ("qkv",)),
    ("gemm_o", ("o_proj", "gemm_o")),
    ("gemm_gate_up", ("gate_up",)),
    ("gemm_down", ("down",)),
    ("gemm_mtp", ("eh_proj",)),
    ("attention", ("attn", "attention", "combine")),
    ("kv_store", ("kv_store", "rope_store", "store_b200", "store_ref")),
    ("norm", ("norm",)),
    ("activation", ("silu", "act")),
    ("collective", COLLECTIVE_NAMES),
    ("embedding", ("embed",)),
    ("lm_head", ("lm_head", "logits", "w8a8")),
    ("sampler", ("argmax", "sample", "greedy", "reject")),
)


def bucket_for(name: str) -> str:
    """Bucket of a range name (the last dotted component is matched first)."""
    low = name.lower()
    leaf = low.rsplit(".", 1)[-1]
    for probe in (leaf, low):
        for bucket, keys in _RULES:
            if any(k in probe for k in keys):
                return bucket
    return "other"


def bucket_kernel(kernel: str, grid_n: int | None = None) -> str:
    """Bucket of a CUDA kernel name (torch.profiler / ncu). Quantized GEMMs
    are told apart by their output width when given (``grid_n`` = N / 128)."""
    k = kernel.lower()
    if "nccl" in k or "multimem" in k or "allreduce" in k:
        return "collective"
    if "decode_attn" in k or "prefill_attn" in k or "decode_combine" in k:
        return "attention"
    if "store_" in k and "kernel" in k:
        return "kv_store"
    if "rmsnorm" in k:
        return "norm"
    if "silu" in k:
        return "activation"
    if "embed" in k:
        return "embedding"
    if "argmax" in k:
        return "sampler"
    if "wq_gemm_kernel<2" in k:
        return "lm_head"
    if "wq_gemm" in k:
        return "gemm"
    return "other"


def exclusive_report(ranges: list[tuple[str, float, float]]) -> dict[str, float]:
    """``ranges`` = (name, start_ms, end_ms) on one stream; properly nested.
    Returns exclusive milliseconds per bucket."""
    out = {b: 0.0 for b in BUCKETS}
    spans = sorted(ranges, key=lambda r: (r[1], -(r[2] - r[1])))
    stack: list[list] = []  # [name, start, end, child_ms]
    def close(node):
        name, s, e, child = node
        out[bucket_for(name)] += max(0.0, (e - s) - child)
        if stack:
            stack[-1][3] += e - s
    for name, s, e in spans:
        while stack and stack[-1][2] <= s:
            close(stack.pop())
        stack.append([name, s, e, 0.0])
    while stack:
        close(stack.pop())
    return out


class _Null(contextlib.AbstractContextManager):
    def __exit__(self, *exc):
        return False


_NULL = _Null()


class StageProfiler:
    def __init__(self, out_dir: str | None = None, rank: int = 0):
        import torch
        self.torch = torch
        self.out_dir = out_dir or os.environ.get("K8V4_PROFILE_DIR", ".")
        self.rank = rank
        self.events: list[tuple[str, object, object]] = []
        self.enabled = True

    @contextlib.contextmanager
    def range(self, name: str):
        torch = self.torch
        if not self.enabled or (torch.cuda.is_available() and torch.cuda.is_current_stream_capturing()):
            yield
            return
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        torch.cuda.nvtx.range_push(name)
        a.record()
        try:
            yield
        finally:
            b.record()
            torch.cuda.nvtx.range_pop()
            self.events.append((name, a, b))

    def collect(self) -> list[tuple[str, float, float]]:
        """(name, start_ms, end_ms) relative to the first event (synchronizes)."""
        if not self.events:
            return []
        self.torch.cuda.synchronize()
        t0 = self.events[0][1]
        return [(n, t0.elapsed_time(a), t0.elapsed_time(b)) for n, a, b in self.events]

    def report(self) -> dict:
        ranges = self.collect()
        return {"rank": self.rank, "pid": os.getpid(), "ranges": len(ranges),
                "exclusive_ms": exclusive_report(ranges), "time": time.time()}

    def write(self, tag: str = "stages") -> str:
        os.makedirs(self.out_dir, exist_ok=True)
        path = os.path.join(self.out_dir, "%s_rank%d_pid%d.json" % (tag, self.rank, os.getpid()))
        with open(path, "w") as f:
            json.dump(self.report(), f, indent=2)
        self.events.clear()
        return path


PROFILER: StageProfiler | None = None


def install(out_dir: str | None = None, rank: int = 0) -> StageProfiler:
    global PROFILER
    PROFILER = StageProfiler(out_dir, rank)
    return PROFILER


def uninstall() -> None:
    global PROFILER
    PROFILER = None


def stage(name: str):
    """Range around one stage; a no-op unless the profiler is installed."""
    p = PROFILER
    return _NULL if p is None else p.range(name)


def install_if_requested(rank: int = 0) -> StageProfiler | None:
    if os.environ.get("K8V4_PROFILE", "0") not in ("", "0", "false"):
        return install(os.environ.get("K8V4_PROFILE_DIR"), rank)
    return None
