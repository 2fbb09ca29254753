"""Host-side batch planning for K8/V4 attention.

Behaviour of the reference's planner (``k8v4_v030/plan.py:22-146``) for the
b200 format:

* ``uniform_packed_q_len`` decides whether a batch is a *uniform packed
  decode*: every request has the same query length, at most the decode
  limit (``128 // gqa`` rows in the b200 decode kernel, i.e. 21 tokens at GQA
  6; the reference used 10). Such a batch runs as one split-K decode launch
  over all requests (and can be replayed from a CUDA graph); anything else is
  prefill;
* ``query_segments`` turns cumulative query offsets into per-request spans;
* ``decode_workspace_floats`` sizes the split-K partial buffers;
* ``require_decoder`` refuses model features the kernels do not implement
  (sliding windows, ALiBi, logit soft-capping, encoder attention, head sizes
  other than 128, KV-head counts the GQA split cannot serve).
"""
from __future__ import annotations

from collections.abc import Sequence

from ..kv.layout import B200_FORMAT, PageLayout

DECODE_MAX_ROWS = 64  # query rows (tokens x GQA) one decode CTA holds


def decode_max_q_len(gqa: int) -> int:
    return DECODE_MAX_ROWS // gqa


def uniform_packed_q_len(query_lens: Sequence[int], gqa: int = 6) -> int | None:
    """The common query length when every request has the same one and it fits
    the decode kernel; ``None`` for a mixed or prefill batch."""
    if not query_lens:
        return None
    q = int(query_lens[0])
    if q < 1 or q > decode_max_q_len(gqa):
        return None
    return q if all(int(x) == q for x in query_lens) else None


def query_segments(cu_q: Sequence[int]) -> list[tuple[int, int]]:
    """(start, end) row span of every request from cumulative offsets."""
    if len(cu_q) < 1 or int(cu_q[0]) != 0:
        raise ValueError("cu_q must start at 0")
    out = []
    for a, b in zip(cu_q[:-1], cu_q[1:]):
        if int(b) < int(a):
            raise ValueError("cu_q must be non-decreasing")
        out.append((int(a), int(b)))
    return out


def decode_workspace_floats(nseq: int, hkv: int, nsplit: int, q_len: int, gqa: int) -> int:
    """fp32 words of the split-K (m, l, O) partials of one decode launch."""
    rows = q_len * gqa
    npad = 16 if rows <= 16 else 32 if rows <= 32 else 48 if rows <= 48 else 64
    return nseq * hkv * nsplit * npad * (128 + 2)


def layout_for_heads(num_heads: int, num_kv_heads: int) -> PageLayout:
    """The b200-format layout of a rank with these local heads."""
    return PageLayout.for_rank(num_heads, num_kv_heads, B200_FORMAT)


def require_decoder(head_size: int, num_heads: int, num_kv_heads: int, sliding_window: int | None = None,
                    alibi_slopes=None, logits_soft_cap: float | None = None, attn_type: str = "decoder",
                    sinks=None) -> PageLayout:
    if attn_type != "decoder":
        raise NotImplementedError("K8/V4 attention serves decoder self-attention only, not %s" % attn_type)
    if head_size != 128:
        raise NotImplementedError("K8/V4 b200 pages hold head_dim 128, got %d" % head_size)
    if sliding_window not in (None, 0, -1):
        raise NotImplementedError("sliding-window attention is not supported")
    if alibi_slopes is not None:
        raise NotImplementedError("ALiBi is not supported")
    if logits_soft_cap not in (None, 0, 0.0):
        raise NotImplementedError("logit soft-capping is not supported")
    if sinks is not None:
        raise NotImplementedError("attention sinks are not supported")
    return layout_for_heads(num_heads, num_kv_heads)
