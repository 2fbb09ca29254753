"""Typed plane views over a K8/V4 byte cache, without copies.

A layer's cache is a byte tensor whose address order is the page order. It
arrives either as ``[num_pages, page_bytes]`` (this framework's own
allocation) or as a vLLM-style logical ``[block, head, token, cell]`` tensor
whose memory order differs from its logical order. The views are built from
the layout's own plane table (``PageLayout.regions``) over the tensor's bytes
in address order, so they work for both. Capability of the reference's
``k8v4_v030/cache_views.py:28-109``: only a tensor whose bytes form one dense,
forward run is accepted, and a head count other than the layout's is refused.
"""
from __future__ import annotations

import torch

from .layout import PageLayout

_TORCH_DTYPE = {"int8": torch.int8, "uint8": torch.uint8, "float32": torch.float32, "float16": torch.float16}
# Plane views start on a 16-byte boundary: the widest element and every TMA
# or bulk copy of a page need no more.
_BASE_ALIGN = 16


def span_problem(t: torch.Tensor) -> str | None:
    """Why ``t``'s bytes are not one dense, forward, non-overlapping run, or
    ``None`` when they are.

    Taking the dimensions longer than 1 from the fastest stride to the
    slowest, each stride must equal the number of bytes the faster ones
    span. That one rule refuses gaps, overlaps (stride 0 or a repeated
    stride) and negative strides alike.
    """
    if t.dtype not in (torch.uint8, torch.int8):
        return "a K8/V4 cache is a byte tensor, got %s" % t.dtype
    if t.numel() == 0:
        return "the K8/V4 cache tensor holds no bytes"
    spanned = 1
    for size, stride in sorted(((n, s) for n, s in zip(t.shape, t.stride()) if n > 1), key=lambda d: d[1]):
        if stride != spanned:
            return ("the K8/V4 cache bytes are not one dense run: a dimension of %d has stride %d where %d "
                    "would continue the run (shape %s, strides %s)"
                    % (size, stride, spanned, tuple(t.shape), tuple(t.stride())))
        spanned *= size
    if t.storage_offset() % _BASE_ALIGN:
        return "the K8/V4 cache starts %d bytes into its storage, not on a %d-byte boundary" % (
            t.storage_offset(), _BASE_ALIGN)
    return None


def byte_run(t: torch.Tensor) -> torch.Tensor:
    """``t``'s bytes as one uint8 vector in address order (shares storage)."""
    why = span_problem(t)
    if why:
        raise RuntimeError(why)
    run = t.as_strided((t.numel(),), (1,), t.storage_offset())
    return run.view(torch.uint8)


def _head_axis_problem(t: torch.Tensor, layout: PageLayout) -> str | None:
    """A vLLM-style ``[block, head, token, cell]`` tensor names its head count
    on axis 1: it must be the layout's, whatever the memory order."""
    if t.dim() == 4 and t.shape[-1] == layout.fmt.slot_bytes_per_head and t.shape[1] != layout.hkv:
        return "the cache tensor holds %d KV heads per block but this rank's layout stores %d" % (
            t.shape[1], layout.hkv)
    return None


def bind_regions(kv_cache: torch.Tensor, layout: PageLayout) -> dict[str, torch.Tensor]:
    """One view per plane (``k``, ``v``, ``k_scale``, ``v_scale`` [, ``v_zero``]),
    indexed ``[page, token, head(, col)]`` and sharing the cache's storage."""
    why = _head_axis_problem(kv_cache, layout)
    if why:
        raise RuntimeError(why)
    run = byte_run(kv_cache)
    pages, rest = divmod(run.numel(), layout.page_bytes)
    if rest:
        raise RuntimeError("%d cache bytes are not a whole number of %d-byte pages" % (run.numel(), layout.page_bytes))
    views: dict[str, torch.Tensor] = {}
    for r in layout.regions:
        typed = run.view(_TORCH_DTYPE[r.dtype])
        e = r.elem
        size = (pages, layout.page, layout.hkv) + ((r.cols,) if r.cols > 1 else ())
        stride = (layout.page_bytes // e, r.token_step // e, r.head_step // e) + ((1,) if r.cols > 1 else ())
        views[r.name] = typed.as_strided(size, stride, (run.storage_offset() + r.offset) // e)
    return views


def allocate_cache(num_pages: int, layout: PageLayout, device="cpu", zero: bool = True) -> torch.Tensor:
    """A ``[num_pages, page_bytes]`` uint8 cache for one layer."""
    shape = (int(num_pages), layout.page_bytes)
    make = torch.zeros if zero else torch.empty
    return make(shape, dtype=torch.uint8, device=device)
