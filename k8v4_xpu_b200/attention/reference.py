"""Eager (torch) paged attention over K8/V4 pages: the dense oracle.

Behaviour of the reference's eager prefill (``k8v4_v030/dequant.py:68-242,
448-501``): gather and dequantize a request's pages per KV head, then

* up to ``SDPA_MAX_KEYS`` keys: one scaled-dot-product attention with a
  bottom-right causal mask (query row i of a q_len-row chunk sees keys
  ``< seq_len - q_len + i + 1``), or explicit per-row ends (MTP trees);
* beyond: a tiled online softmax that gathers each key tile once, bounding
  the score tile to ``SCORE_TILE_BYTES``.

Runs on CPU or GPU tensors; the gather is the torch one on CPU and the
``k8v4.gather_dequant`` kernel on a CUDA cache. It is the reference the
CUDA kernels are tested against at long contexts, and the public
``paged_prefill`` / ``eager_prefill`` API of the attention package.
"""
from __future__ import annotations

import math

import torch

from ..kv.layout import PageLayout, b200_layout

SDPA_MAX_KEYS = 16384
SCORE_TILE_BYTES = 128 << 20


def gather_dequant_head(cache: torch.Tensor, pages: list[int] | torch.Tensor, seq_len: int, layout: PageLayout,
                        head: int) -> tuple[torch.Tensor, torch.Tensor]:
    """fp32 ``[seq_len, 128]`` K and V of one KV head."""
    if cache.is_cuda:
        from .. import ops
        bt = torch.as_tensor(pages, dtype=torch.int32, device=cache.device)
        return ops.gather_dequant(cache, bt, layout.hkv, head, seq_len)
    from ..kv.pack import gather_sequence
    k, v = gather_sequence(cache, list(torch.as_tensor(pages).tolist()), seq_len, layout)
    return k[:, head].contiguous(), v[:, head].contiguous()


def _ends(seq_len: int, q_len: int, q_ends) -> torch.Tensor:
    if q_ends is not None:
        return torch.as_tensor(q_ends, dtype=torch.int64)
    return torch.arange(q_len, dtype=torch.int64) + (seq_len - q_len + 1)


def attention_dense(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, ends: torch.Tensor, scale: float,
                    quant_q: bool = False) -> torch.Tensor:
    """q [Tq, G, D] (the GQA rows of one KV head), k/v [S, D]; row t sees keys < ends[t]."""
    Tq, G, D = q.shape
    S = k.shape[0]
    qf = q.float()
    if quant_q:  # the kernels' int8 Q with a per-row fp32 scale
        from ..kv.oracle import quant_k_t
        q8, qs = quant_k_t(qf, "float32")
        qf = q8.float() * qs.unsqueeze(-1)
    dev = q.device
    if S <= SDPA_MAX_KEYS:
        scores = torch.einsum("tgd,sd->tgs", qf, k.float()) * scale
        mask = torch.arange(S, device=dev).view(1, 1, S) >= ends.to(dev).view(Tq, 1, 1)
        scores = scores.masked_fill(mask, float("-inf"))
        p = torch.softmax(scores, -1).nan_to_num(0.0)
        return torch.einsum("tgs,sd->tgd", p, v.float())
    # tiled online softmax: each key tile gathered once
    tile = max(256, SCORE_TILE_BYTES // max(1, Tq * G * 4))
    m = torch.full((Tq, G), float("-inf"), device=dev)
    l = torch.zeros((Tq, G), device=dev)
    acc = torch.zeros((Tq, G, D), device=dev)
    for s0 in range(0, S, tile):
        kt, vt = k[s0:s0 + tile].float(), v[s0:s0 + tile].float()
        sc = torch.einsum("tgd,sd->tgs", qf, kt) * scale
        idx = torch.arange(s0, s0 + kt.shape[0], device=dev).view(1, 1, -1)
        sc = sc.masked_fill(idx >= ends.to(dev).view(Tq, 1, 1), float("-inf"))
        mn = torch.maximum(m, sc.amax(-1))
        safe = torch.where(torch.isfinite(mn), mn, torch.zeros_like(mn))
        a = torch.exp(m - safe).nan_to_num(0.0)
        p = torch.exp(sc - safe.unsqueeze(-1)).nan_to_num(0.0)
        l = l * a + p.sum(-1)
        acc = acc * a.unsqueeze(-1) + torch.einsum("tgs,sd->tgd", p, vt)
        m = mn
    return acc / torch.where(l > 0, l, torch.ones_like(l)).unsqueeze(-1)


def eager_prefill(q: torch.Tensor, cache: torch.Tensor, pages, seq_len: int, hkv: int, gqa: int,
                  scale: float | None = None, q_ends=None, quant_q: bool = False) -> torch.Tensor:
    """One request: q [q_len, hkv*gqa, 128] -> out [q_len, hkv*gqa, 128] fp32."""
    layout = b200_layout(hkv, gqa)
    q_len = q.shape[0]
    scale = 1.0 / math.sqrt(q.shape[-1]) if scale is None else scale
    ends = _ends(seq_len, q_len, q_ends)
    out = torch.empty(q.shape, dtype=torch.float32, device=q.device)
    for h in range(hkv):
        k, v = gather_dequant_head(cache, pages, seq_len, layout, h)
        out[:, h * gqa:(h + 1) * gqa] = attention_dense(q[:, h * gqa:(h + 1) * gqa], k.to(q.device),
                                                        v.to(q.device), ends, scale, quant_q)
    return out


def paged_prefill(q: torch.Tensor, cache: torch.Tensor, block_table: torch.Tensor, seq_lens: torch.Tensor,
                  cu_q: torch.Tensor, hkv: int, gqa: int, scale: float | None = None) -> torch.Tensor:
    """Batched paged causal prefill (head-major API of the reference,
    ``onednn_prefill.py:188-241``): the ``k8v4.prefill_attn`` kernel on a CUDA
    cache, this module's eager path elsewhere."""
    max_q = int((cu_q[1:] - cu_q[:-1]).max().item())
    if cache.is_cuda:
        from .. import ops
        return ops.prefill_attn(q, cu_q, seq_lens, block_table, cache, hkv, gqa, max_q, sm_scale=scale)
    out = torch.empty(q.shape, dtype=torch.float32)
    cu = cu_q.tolist()
    for b in range(len(cu) - 1):
        n = int(seq_lens[b])
        npg = (n + 15) // 16
        out[cu[b]:cu[b + 1]] = eager_prefill(q[cu[b]:cu[b + 1]], cache, block_table[b, :npg], n, hkv, gqa, scale)
    return out.to(q.dtype)
