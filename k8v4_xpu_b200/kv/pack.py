"""Byte-level pack and unpack of K8/V4 pages (CPU reference of the store kernel).

``write_token`` / ``read_token`` work on a ``bytearray`` one token at a time
(behaviour of ``k8v4_v030/paged.py:30-91``); ``store_tokens`` and
``gather_sequence`` are the vectorized torch equivalents used as oracles for
the CUDA store and gather kernels. A negative slot is a no-op everywhere.
"""
from __future__ import annotations

import struct

import torch

from .layout import PageLayout, kernel_page_and_offset
from .oracle import (
    dequant_k_t,
    dequant_v_affine_t,
    dequant_v_sym_t,
    pack_nibbles,
    quant_k_t,
    quant_v_affine_t,
    quant_v_sym_t,
    unpack_nibbles,
)
from .views import bind_regions

_FMT = {"float32": "<f", "float16": "<e"}


def _put_scale(blob: bytearray, at: int, value: float, sdt: str) -> None:
    n = 4 if sdt == "float32" else 2
    blob[at:at + n] = struct.pack(_FMT[sdt], value)


def _get_scale(blob: bytearray, at: int, sdt: str) -> float:
    n = 4 if sdt == "float32" else 2
    return struct.unpack(_FMT[sdt], bytes(blob[at:at + n]))[0]


def write_token(blob: bytearray, slot: int, keys, values, layout: PageLayout) -> None:
    """Quantize one token (``[HKV][D]`` floats) into the page that owns ``slot``."""
    page, off = kernel_page_and_offset(slot, layout.page)
    if page < 0:
        return
    if len(keys) != layout.hkv or len(values) != layout.hkv:
        raise ValueError("expected %d KV heads" % layout.hkv)
    if len(blob) < (page + 1) * layout.page_bytes:
        raise ValueError("blob shorter than page %d" % page)
    fmt = layout.fmt
    k = torch.tensor(keys, dtype=torch.float32)
    v = torch.tensor(values, dtype=torch.float32)
    kq, ks = quant_k_t(k, fmt.scale_dtype)
    for head in range(layout.hkv):
        base = layout.byte_of("k", page, off, head)
        blob[base:base + fmt.head_dim] = kq[head].numpy().tobytes()
        _put_scale(blob, layout.byte_of("k_scale", page, off, head), float(ks[head]), fmt.scale_dtype)
        if fmt.v_mode == "affine_row":
            nib, vs, vz = quant_v_affine_t(v[head])
            _put_scale(blob, layout.byte_of("v_scale", page, off, head), float(vs), fmt.scale_dtype)
            _put_scale(blob, layout.byte_of("v_zero", page, off, head), float(vz), fmt.scale_dtype)
        else:
            nib, vs = quant_v_sym_t(v[head], fmt.v_group)
            for g in range(fmt.v_groups):
                at = layout.byte_of("v_scale", page, off, head, g)
                _put_scale(blob, at, float(vs[g]), fmt.scale_dtype)
        vb = layout.byte_of("v", page, off, head)
        blob[vb:vb + fmt.v_cols] = pack_nibbles(nib).numpy().tobytes()


def read_token(blob: bytearray, slot: int, layout: PageLayout):
    """Dequantize one stored token; inverse of ``write_token`` up to rounding."""
    page, off = kernel_page_and_offset(slot, layout.page)
    if page < 0:
        raise ValueError("negative slot")
    fmt = layout.fmt
    keys, values = [], []
    for head in range(layout.hkv):
        base = layout.byte_of("k", page, off, head)
        kq = torch.frombuffer(bytearray(blob[base:base + fmt.head_dim]), dtype=torch.int8)
        ks = _get_scale(blob, layout.byte_of("k_scale", page, off, head), fmt.scale_dtype)
        keys.append((kq.float() * ks).tolist())
        vb = layout.byte_of("v", page, off, head)
        nib = unpack_nibbles(torch.frombuffer(bytearray(blob[vb:vb + fmt.v_cols]), dtype=torch.uint8))
        if fmt.v_mode == "affine_row":
            vs = _get_scale(blob, layout.byte_of("v_scale", page, off, head), fmt.scale_dtype)
            vz = _get_scale(blob, layout.byte_of("v_zero", page, off, head), fmt.scale_dtype)
            values.append(((nib.float() - vz) * vs).tolist())
        else:
            scales = torch.tensor([_get_scale(blob, layout.byte_of("v_scale", page, off, head, g),
                                              fmt.scale_dtype) for g in range(fmt.v_groups)])
            values.append(dequant_v_sym_t(nib, scales, fmt.v_group).tolist())
    return keys, values


# --------------------------------------------------------------- vectorized


def store_tokens(cache: torch.Tensor, slots: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                 layout: PageLayout) -> None:
    """Quantize ``k``/``v`` ``[T, HKV, D]`` into ``cache`` at ``slots`` (torch reference).

    Slots that are negative or past the cache are skipped, like the kernel.
    """
    regions = bind_regions(cache, layout)
    fmt = layout.fmt
    num_pages = regions["k"].shape[0]
    slots = slots.to(torch.int64).cpu()
    keep = (slots >= 0) & (slots < num_pages * layout.page)
    if not bool(keep.any()):
        return
    idx = keep.nonzero().flatten()
    s = slots[idx]
    pg, off = s // layout.page, s % layout.page
    kk = k[idx].float()
    vv = v[idx].float()
    kq, ks = quant_k_t(kk, fmt.scale_dtype)
    regions["k"][pg, off] = kq
    regions["k_scale"][pg, off] = ks
    if fmt.v_mode == "affine_row":
        nib, vs, vz = quant_v_affine_t(vv)
        regions["v_scale"][pg, off] = vs.to(regions["v_scale"].dtype)
        regions["v_zero"][pg, off] = vz.to(regions["v_zero"].dtype)
    else:
        nib, vs = quant_v_sym_t(vv, fmt.v_group)
        regions["v_scale"][pg, off] = vs
    regions["v"][pg, off] = pack_nibbles(nib)


def gather_sequence(cache: torch.Tensor, page_ids, seq_len: int, layout: PageLayout):
    """Dequantized ``(k, v)`` ``[seq_len, HKV, D]`` fp32 of one sequence's pages."""
    regions = bind_regions(cache, layout)
    fmt = layout.fmt
    pages = torch.as_tensor(list(page_ids), dtype=torch.int64)
    n_pages = (int(seq_len) + layout.page - 1) // layout.page
    pages = pages[:n_pages]
    kq = regions["k"][pages].reshape(-1, layout.hkv, fmt.head_dim)[:seq_len]
    ks = regions["k_scale"][pages].reshape(-1, layout.hkv)[:seq_len]
    vp = regions["v"][pages].reshape(-1, layout.hkv, fmt.v_cols)[:seq_len]
    nib = unpack_nibbles(vp)
    k = dequant_k_t(kq, ks)
    if fmt.v_mode == "affine_row":
        vs = regions["v_scale"][pages].reshape(-1, layout.hkv)[:seq_len]
        vz = regions["v_zero"][pages].reshape(-1, layout.hkv)[:seq_len]
        v = dequant_v_affine_t(nib, vs, vz)
    else:
        vs = regions["v_scale"][pages].reshape(-1, layout.hkv, fmt.v_groups)[:seq_len]
        v = dequant_v_sym_t(nib, vs, fmt.v_group)
    return k, v
