"""Typed region views over a K8/V4 byte cache, without copies.

The cache of one layer is a byte tensor whose address order is the page
order. It can arrive as ``[num_pages, page_bytes]`` (this framework's own
allocation) or as a vLLM-style logical ``[block, head, token, cell]`` tensor
whose memory order differs from its logical order. Either way the bytes must
form one dense span; a gapped, overlapping or negatively strided tensor is
refused (behaviour of ``k8v4_v030/cache_views.py:28-109``).
"""
from __future__ import annotations

import torch

from .layout import PageLayout, region_view_specs

_BYTE = (torch.uint8, torch.int8)
_DT = {"int8": torch.int8, "uint8": torch.uint8, "float32": torch.float32, "float16": torch.float16}


def _dense_reason(kv_cache: torch.Tensor) -> str:
    return "K8/V4 layer cache is not a dense byte span (shape=%s stride=%s)" % (
        tuple(kv_cache.shape), tuple(kv_cache.stride()))


def memory_order_bytes(kv_cache: torch.Tensor) -> torch.Tensor:
    """One uint8 vector of ``kv_cache`` in address order (no copy)."""
    if kv_cache.dtype not in _BYTE:
        raise RuntimeError("K8/V4 cache dtype %s is not a byte tensor" % kv_cache.dtype)
    if kv_cache.numel() == 0:
        raise RuntimeError("K8/V4 cache tensor is empty")
    dims = [(int(n), int(s)) for n, s in zip(kv_cache.shape, kv_cache.stride()) if int(n) != 1]
    for _n, s in dims:
        if s <= 0:
            raise RuntimeError(_dense_reason(kv_cache))
    covered = 1
    for n, s in sorted(dims, key=lambda item: item[1]):
        if s != covered:
            raise RuntimeError(_dense_reason(kv_cache))
        covered *= n
    if covered != int(kv_cache.numel()):
        raise RuntimeError(_dense_reason(kv_cache))
    base = int(kv_cache.storage_offset())
    if base % 16 != 0:
        raise RuntimeError("K8/V4 cache storage is not 16-byte aligned")
    flat = torch.as_strided(kv_cache, size=(int(kv_cache.numel()),), stride=(1,), storage_offset=base)
    return flat if flat.dtype == torch.uint8 else flat.view(torch.uint8)


def bind_regions(kv_cache: torch.Tensor, layout: PageLayout) -> dict[str, torch.Tensor]:
    """Region views (``k``, ``v``, ``k_scale``, ``v_scale`` [, ``v_zero``]) sharing storage."""
    if kv_cache.dim() == 4 and kv_cache.shape[1] > 1 and kv_cache.shape[1] != layout.hkv:
        raise RuntimeError("K8/V4 cache has %d KV heads, layout serves %d"
                           % (int(kv_cache.shape[1]), layout.hkv))
    raw = memory_order_bytes(kv_cache)
    if raw.numel() % layout.page_bytes != 0:
        raise RuntimeError("K8/V4 cache has %d bytes, not a multiple of the %d-byte page"
                           % (raw.numel(), layout.page_bytes))
    num_pages = raw.numel() // layout.page_bytes
    specs = region_view_specs(num_pages, layout)
    base = int(raw.storage_offset())
    views: dict[str, torch.Tensor] = {}
    for name, spec in specs.items():
        dt = _DT[str(spec["dtype"])]
        storage = raw.view(dt)
        esz = storage.element_size()
        off = base + int(spec["byte_offset"])
        if off % esz:
            raise RuntimeError("region %s misaligned for %s" % (name, dt))
        views[name] = torch.as_strided(storage, size=spec["shape"], stride=spec["stride"],
                                       storage_offset=off // esz)
    return views


def allocate_cache(num_pages: int, layout: PageLayout, device="cpu", zero: bool = True) -> torch.Tensor:
    """A ``[num_pages, page_bytes]`` uint8 cache for one layer."""
    shape = (int(num_pages), layout.page_bytes)
    if zero:
        return torch.zeros(shape, dtype=torch.uint8, device=device)
    return torch.empty(shape, dtype=torch.uint8, device=device)
