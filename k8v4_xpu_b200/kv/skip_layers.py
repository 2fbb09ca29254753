"""Per-layer KV cache dtype override: "skip layers" keep a plain fp8 or bf16
paged cache next to the K8/V4 layers.

Reference behaviour (``tools/patch_vllm_skip_fp8.py:1-188``): the layers
listed in ``kv_cache_dtype_skip_layers`` take the dtype that
``VLLM_KV_SKIP_DTYPE`` names (default ``auto``, the model dtype) instead of
K8/V4 and run the stock attention backend (``:62-70``, ``:123-140``). In
vLLM all KV groups share one page size, so a skipped layer's page is padded
up to the K8/V4 page, its block is the largest 64-token multiple that divides
that page with a 16-byte token stride, and the padding is spread over the
tokens (``:47-61``, ``:81-117``, ``:160-186``).

Here every layer's cache is its own tensor indexed by the same page ids, so a
skip layer needs neither a second block table nor padding: its page holds the
same 16 tokens as a K8/V4 page, each token ``[K | V]`` over the KV heads in
the skip dtype (``2 * hkv * head_dim * itemsize`` bytes, a multiple of 16),
and the capacity fit counts the wider page (:func:`pool_bytes_per_page`). One
extra page at the end of the tensor takes the writes of padding rows (slot
-1), so the store has no branch and no read-modify-write.

The skip layers' attention is the framework's torch path (no K8/V4 kernel
reads these pages): a key-tiled online softmax over the block table with the
K8/V4 kernels' bottom-right causal rule (row ``t`` sees keys
``< positions[t] + 1``, or ``< q_ends[t]``). Its shapes depend only on the
batch's static sizes, so a decode step that holds it can be captured in a CUDA
graph; outside a capture the key range is trimmed to the longest sequence.
Every gathered index is clamped into the pool, so stale metadata cannot make
the gather leave the tensor. fp8 K and V use one scale per layer (1.0 unless
given), the stock fp8 KV convention. Gathers and stores move raw bytes
(``uint8``) and reinterpret them, so no indexing kernel needs a float8 type.
"""
from __future__ import annotations

import dataclasses
import math
import os
from typing import Mapping

import torch

from .layout import B200_FORMAT

# name -> storage dtype ("auto": the model's compute dtype, bf16 here)
SKIP_DTYPES: dict[str, torch.dtype] = {
    "auto": torch.bfloat16,
    "bfloat16": torch.bfloat16,
    "fp8": torch.float8_e4m3fn,
    "fp8_e4m3": torch.float8_e4m3fn,
    "fp8_e5m2": torch.float8_e5m2,
}
# this framework's variable first, then the reference deployment's name
SKIP_DTYPE_ENV = ("K8V4_KV_SKIP_DTYPE", "VLLM_KV_SKIP_DTYPE")
SCORE_TILE_BYTES = 128 << 20


def resolve_skip_dtype(name: str | None = None, env: Mapping[str, str] | None = None) -> str:
    """The skip layers' dtype name: ``name`` if given, else the first set
    variable of :data:`SKIP_DTYPE_ENV`, else ``auto``. Raises on unknown names."""
    if name is None:
        env = os.environ if env is None else env
        name = next((env[v] for v in SKIP_DTYPE_ENV if env.get(v)), "auto")
    name = name.strip().lower()
    if name not in SKIP_DTYPES:
        raise ValueError("unknown skip-layer KV dtype %r (one of %s)" % (name, ", ".join(sorted(SKIP_DTYPES))))
    return name


def parse_layers(spec) -> tuple[int, ...]:
    """``"0,3,7"`` / ``[0, 3, 7]`` / ``None`` -> sorted unique layer indices."""
    if spec is None:
        return ()
    if isinstance(spec, str):
        spec = [s for s in spec.replace(" ", "").split(",") if s]
    out = sorted({int(s) for s in spec})
    if out and out[0] < 0:
        raise ValueError("skip-layer indices must be non-negative: %s" % out)
    return tuple(out)


def _fp8_max(dtype: torch.dtype) -> float | None:
    return torch.finfo(dtype).max if dtype in (torch.float8_e4m3fn, torch.float8_e5m2) else None


@dataclasses.dataclass(frozen=True)
class SkipLayout:
    """Page geometry of one skip layer's cache (one TP rank's KV heads)."""

    hkv: int
    dtype_name: str = "auto"
    head_dim: int = B200_FORMAT.head_dim
    page: int = B200_FORMAT.page
    k_scale: float = 1.0
    v_scale: float = 1.0

    def __post_init__(self) -> None:
        resolve_skip_dtype(self.dtype_name)
        if self.hkv < 1 or self.head_dim < 1 or self.page < 1:
            raise ValueError("skip layout needs positive heads, head_dim and page")
        if self.token_bytes % 16:
            raise ValueError("token stride %d is not a multiple of 16 bytes" % self.token_bytes)

    @property
    def dtype(self) -> torch.dtype:
        return SKIP_DTYPES[self.dtype_name]

    @property
    def itemsize(self) -> int:
        return torch.empty((), dtype=self.dtype).element_size()

    @property
    def half_bytes(self) -> int:
        """Bytes of K (or V) of one token: every KV head."""
        return self.hkv * self.head_dim * self.itemsize

    @property
    def token_bytes(self) -> int:
        return 2 * self.half_bytes

    @property
    def page_bytes(self) -> int:
        return self.page * self.token_bytes

    def alloc(self, num_pages: int, device="cpu") -> torch.Tensor:
        """Zeroed ``uint8 [num_pages + 1, page_bytes]``; the last page is the
        sink for padding rows' writes and is never handed out."""
        return torch.zeros((num_pages + 1, self.page_bytes), dtype=torch.uint8, device=device)

    def token_rows(self, pool: torch.Tensor) -> torch.Tensor:
        """``uint8 [pages * page, token_bytes]``: one row per token slot."""
        return pool.view(pool.shape[0] * self.page, self.token_bytes)

    def decode(self, raw: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        """fp32 K and V ``[..., hkv, head_dim]`` of token rows ``[..., token_bytes]``."""
        lead = raw.shape[:-1]
        k = raw[..., : self.half_bytes].contiguous().view(self.dtype).view(*lead, self.hkv, self.head_dim)
        v = raw[..., self.half_bytes:].contiguous().view(self.dtype).view(*lead, self.hkv, self.head_dim)
        return k.float() * self.k_scale, v.float() * self.v_scale

    def encode(self, k: torch.Tensor, v: torch.Tensor) -> torch.Tensor:
        """Token rows ``uint8 [T, token_bytes]`` of K and V ``[T, hkv, head_dim]``."""
        T = k.shape[0]

        def q(x: torch.Tensor, scale: float) -> torch.Tensor:
            x = x.float()
            if scale != 1.0:
                x = x / scale
            lim = _fp8_max(self.dtype)
            if lim is not None:
                x = x.clamp(-lim, lim)
            return x.to(self.dtype).reshape(T, -1).view(torch.uint8)

        return torch.cat([q(k, self.k_scale), q(v, self.v_scale)], dim=1)


def pool_bytes_per_page(k8v4_page_bytes: int, n_layers: int, skip: Mapping[int, SkipLayout]) -> int:
    """KV bytes one page id costs over every layer (the capacity fit's unit)."""
    return k8v4_page_bytes * (n_layers - len(skip)) + sum(s.page_bytes for s in skip.values())


def store(pool: torch.Tensor, lay: SkipLayout, slots: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> None:
    """Write K/V ``[T, hkv, head_dim]`` of ``T`` tokens at ``slots`` (-1: dropped
    into the sink page)."""
    rows = lay.token_rows(pool)
    sink = rows.shape[0] - 1
    s = slots.to(torch.int64)
    idx = torch.where(s >= 0, s, torch.full_like(s, sink)).clamp(max=sink)
    rows.index_copy_(0, idx, lay.encode(k, v))


def apply_rope(x: torch.Tensor, cos_sin: torch.Tensor, positions: torch.Tensor) -> torch.Tensor:
    """Half-split rotary embedding of ``x [T, h, D]`` with the model's table
    (``[max_pos, D]``: cos of the D/2 frequencies, then their sin), rounded
    to ``x``'s dtype like the fused store kernel's output."""
    D = x.shape[-1]
    pos = positions.to(torch.int64).clamp(0, cos_sin.shape[0] - 1)
    c = cos_sin[pos, : D // 2].unsqueeze(1)
    s = cos_sin[pos, D // 2:].unsqueeze(1)
    a, b = x[..., : D // 2].float(), x[..., D // 2:].float()
    return torch.cat([a * c - b * s, b * c + a * s], -1).to(x.dtype)


def paged_attention(q: torch.Tensor, pool: torch.Tensor, lay: SkipLayout, block_table: torch.Tensor,
                    seq_lens: torch.Tensor, cu_q: torch.Tensor, positions: torch.Tensor, max_q: int, gqa: int,
                    scale: float | None = None, q_ends: torch.Tensor | None = None,
                    score_bytes: int = SCORE_TILE_BYTES) -> torch.Tensor:
    """Causal GQA attention of ``q [T, hkv*gqa, D]`` over a skip layer's pages.

    ``block_table [B, W]`` holds page ids, ``cu_q [B+1]`` the rows of each
    sequence (at most ``max_q``), ``seq_lens [B]`` its keys including these
    rows. Returns ``[T, hkv*gqa, D]`` in ``q``'s dtype; a row that sees no key
    is zero.
    """
    T, hq, D = q.shape
    hkv = lay.hkv
    if hq != hkv * gqa or D != lay.head_dim:
        raise ValueError("q [%d, %d, %d] does not match %d KV heads x %d (D %d)" % (T, hq, D, hkv, gqa, lay.head_dim))
    B, W = block_table.shape
    P = lay.page
    dev = q.device
    scale = 1.0 / math.sqrt(D) if scale is None else scale
    if not (q.is_cuda and torch.cuda.is_current_stream_capturing()) and B > 0:
        # eager: only the pages the longest sequence uses
        W = max(1, min(W, (int(seq_lens.max().item()) + P - 1) // P))
    if T == 0 or B == 0:
        return torch.zeros_like(q)
    cu = cu_q.to(device=dev, dtype=torch.int64)
    qlen = cu[1:] - cu[:-1]
    r = torch.arange(max_q, device=dev)
    valid = r.view(1, -1) < qlen.view(-1, 1)                               # [B, Q]
    tok = (cu[:-1].view(-1, 1) + r.view(1, -1)).clamp(0, T - 1)          # [B, Q]
    ends = (q_ends.to(torch.int64) if q_ends is not None else positions.to(torch.int64) + 1)[tok]
    ends = torch.where(valid, ends, torch.zeros_like(ends))              # [B, Q]
    qp = q[tok].float().view(B, max_q, hkv, gqa, D) * scale
    lens = seq_lens.to(device=dev, dtype=torch.int64).view(B, 1)
    sink = pool.shape[0] - 1
    m = torch.full((B, max_q, hkv, gqa), float("-inf"), device=dev)
    l = torch.zeros((B, max_q, hkv, gqa), device=dev)
    acc = torch.zeros((B, max_q, hkv, gqa, D), device=dev)
    per_key = B * max_q * hq * 4 * 2 + B * lay.token_bytes * 5
    pages_per_tile = max(1, score_bytes // max(1, per_key * P))
    for p0 in range(0, W, pages_per_tile):
        bt = block_table[:, p0:min(W, p0 + pages_per_tile)].to(torch.int64).clamp(0, sink)
        n = bt.shape[1] * P
        raw = pool[bt].view(B, n, lay.token_bytes)
        kt, vt = lay.decode(raw)                                           # [B, n, hkv, D]
        key = torch.arange(p0 * P, p0 * P + n, device=dev)
        live = (key.view(1, n) < lens).view(B, n, 1, 1)
        kt = torch.where(live, kt, torch.zeros_like(kt))
        vt = torch.where(live, vt, torch.zeros_like(vt))
        sc = torch.einsum("bqhgd,bnhd->bqhgn", qp, kt)
        hide = key.view(1, 1, 1, 1, n) >= ends.view(B, max_q, 1, 1, 1)
        sc = sc.masked_fill(hide, float("-inf"))
        mn = torch.maximum(m, sc.amax(-1))
        safe = torch.where(torch.isfinite(mn), mn, torch.zeros_like(mn))
        a = torch.exp(m - safe)
        p = torch.exp(sc - safe.unsqueeze(-1))
        l = l * a + p.sum(-1)
        acc = acc * a.unsqueeze(-1) + torch.einsum("bqhgn,bnhd->bqhgd", p, vt)
        m = mn
    out = (acc / torch.where(l > 0, l, torch.ones_like(l)).unsqueeze(-1)).view(B, max_q, hq, D)
    # back to token order: token t is row t - cu[b] of sequence b
    t = torch.arange(T, device=dev)
    seq = torch.searchsorted(cu[1:].contiguous(), t, right=True).clamp(0, B - 1)
    row = (t - cu[seq]).clamp(0, max_q - 1)
    return out[seq, row].to(q.dtype)
