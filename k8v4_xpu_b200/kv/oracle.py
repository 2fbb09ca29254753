"""CPU quantization rules and causal GQA references for the K8/V4 kernels.

Rules (the CUDA store kernel implements exactly these fp32 operations, so
stored bytes match bit for bit):

K, both formats
    symmetric int8 per token per head: ``scale = amax / 127`` (fp32, then cast
    to the format's scale dtype), ``inv = 1 / scale`` computed from the *stored*
    scale, ``q = clamp(rint(x * inv), -127, 127)``. ``rint`` rounds half to even
    (the reference kernel's ``sycl::rint``, ``xe2_kv_ops.cpp:553-571``; its
    Python oracle rounded half away from zero, ``oracle.py:18-19`` -- ties are
    measure-zero and this build defines half-to-even everywhere).

V, ``ref`` format (``oracle.py:47-69``)
    affine uint4 per token per head: ``scale = max((hi-lo)/15, 1e-8)``,
    ``zero = clamp(floor(-lo/scale + 0.5), 0, 15)``,
    ``q = clamp(floor(x/scale + zero + 0.5), 0, 15)``; low nibble = even dim.

V, ``b200`` format
    symmetric int4 with one fp16 scale per 32-element group along head_dim:
    ``scale = amax_group / 7``, ``q = clamp(rint(x * (1/scale)), -7, 7)``,
    stored as the nibble ``q + 8``; low nibble = even dim.

Scores are ``dot(q8, k8) * q_scale * k_scale / sqrt(head_dim)`` with the query
quantized per (token, head) row like K (fp32 scale), matching the decode
kernel's Q-once quantization (``xe2_kv_ops.cpp:205-257``).
"""
from __future__ import annotations

import math

import torch

from .layout import D, REF_FORMAT, PageLayout, builtin_q_end, ref_layout

# ------------------------------------------------------------ scalar (lists)
# Python-list entry points for the reference format. Each one converts to
# tensors, runs the tensor oracle below and converts back, so there is one
# implementation of every rule.


def _row(values, what: str) -> torch.Tensor:
    t = torch.tensor(values, dtype=torch.float32)
    if t.shape != (D,):
        raise ValueError("a reference-format %s row holds %d values, got shape %s" % (what, D, tuple(t.shape)))
    return t


def quant_k(row: list[float]) -> tuple[list[int], float]:
    """Reference-format K row: int8 codes and the fp32 scale."""
    q, s = quant_k_t(_row(row, "K"), "float32")
    return q.tolist(), float(s)


def dequant_k(packed: list[int], scale: float) -> list[float]:
    return dequant_k_t(torch.tensor(packed), torch.tensor(scale)).tolist()


def quant_v(row: list[float]) -> tuple[list[int], float, float]:
    """Reference-format V row: packed affine uint4 bytes (low nibble = even
    dim), scale and zero point."""
    nib, s, z = quant_v_affine_t(_row(row, "V"))
    return pack_nibbles(nib).tolist(), float(s), float(z)


def dequant_v(packed: list[int], scale: float, zero: float) -> list[float]:
    nib = unpack_nibbles(torch.tensor(packed, dtype=torch.uint8))
    return dequant_v_affine_t(nib, torch.tensor(scale), torch.tensor(zero)).tolist()


def causal_gqa(query, key, value, seq_len: int, q_len: int):
    """Quantized causal GQA over Python lists, reference format.

    ``query`` is ``[q_len][HQ][D]`` (the last ``q_len`` tokens of the
    sequence), ``key`` and ``value`` ``[>= seq_len][HKV][D]`` floats, which
    go through the store rules first. Returns ``[q_len][HQ][D]``. The same
    computation as ``attention_ref`` (behaviour of
    ``k8v4_v030/oracle.py:100-163``).
    """
    if int(q_len) == 0:
        if len(query):
            raise ValueError("q_len 0 with %d query rows" % len(query))
        return []
    q = torch.tensor(query, dtype=torch.float32)
    if q.dim() != 3 or q.shape[0] != q_len or q.shape[2] != D:
        raise ValueError("query must be [%d][HQ][%d], got %s" % (q_len, D, tuple(q.shape)))
    k = torch.tensor(key, dtype=torch.float32)
    v = torch.tensor(value, dtype=torch.float32)
    if k.shape[0] < seq_len or v.shape[0] < seq_len or k.shape[1:] != v.shape[1:]:
        raise ValueError("key/value must hold at least %d tokens of the same heads" % seq_len)
    layout = PageLayout.for_rank(q.shape[1], k.shape[1], REF_FORMAT)
    kd, vd = quant_dequant_kv(k[:seq_len], v[:seq_len], layout)
    ends = [builtin_q_end(seq_len, q_len, r) for r in range(q_len)]
    return attention_ref(q, kd, vd, ends, layout.gqa).tolist()


def deterministic_rows(n: int, heads: int, seed: int, dim: int = D):
    """``[n][heads][dim]`` floats, uniform in [-1, 1), reproducible from ``seed``."""
    gen = torch.Generator().manual_seed(int(seed))
    return (torch.rand(n, heads, dim, generator=gen, dtype=torch.float64) * 2.0 - 1.0).tolist()


# ------------------------------------------------------------ torch (tensors)

_SDT = {"float32": torch.float32, "float16": torch.float16}


def quant_k_t(x: torch.Tensor, scale_dtype: str = "float16") -> tuple[torch.Tensor, torch.Tensor]:
    """Symmetric int8 over the last dim. Returns (int8 codes, scale)."""
    x = x.float()
    amax = x.abs().amax(dim=-1)
    scale = (amax / 127.0).to(_SDT[scale_dtype])
    sf = scale.float()
    inv = torch.where(sf > 0, 1.0 / sf, torch.zeros_like(sf))
    q = torch.round(x * inv.unsqueeze(-1)).clamp_(-127, 127).to(torch.int8)
    return q, scale


def dequant_k_t(q: torch.Tensor, scale: torch.Tensor) -> torch.Tensor:
    return q.float() * scale.float().unsqueeze(-1)


def quant_v_affine_t(x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Affine uint4 over the last dim (reference rule). Returns nibbles (int64), scale, zero."""
    x = x.float()
    lo = x.amin(dim=-1)
    hi = x.amax(dim=-1)
    scale = torch.clamp((hi - lo) / 15.0, min=1.0e-8)
    zero = torch.floor(-lo / scale + 0.5).clamp_(0, 15)
    q = torch.floor(x / scale.unsqueeze(-1) + zero.unsqueeze(-1) + 0.5).clamp_(0, 15)
    return q.to(torch.int64), scale, zero


def quant_v_sym_t(x: torch.Tensor, group: int = 32) -> tuple[torch.Tensor, torch.Tensor]:
    """Symmetric int4 per ``group`` elements. Returns nibbles (q+8, int64) and fp16 scales."""
    x = x.float()
    shp = x.shape
    g = x.reshape(*shp[:-1], shp[-1] // group, group)
    amax = g.abs().amax(dim=-1)
    scale = (amax / 7.0).to(torch.float16)
    sf = scale.float()
    inv = torch.where(sf > 0, 1.0 / sf, torch.zeros_like(sf))
    q = torch.round(g * inv.unsqueeze(-1)).clamp_(-7, 7)
    return (q + 8).to(torch.int64).reshape(shp), scale


def pack_nibbles(nib: torch.Tensor) -> torch.Tensor:
    """``[..., D]`` nibbles -> ``[..., D/2]`` uint8, low nibble = even dim."""
    return (nib[..., 0::2] | (nib[..., 1::2] << 4)).to(torch.uint8)


def unpack_nibbles(packed: torch.Tensor) -> torch.Tensor:
    p = packed.to(torch.int64)
    out = torch.stack([p & 0xF, p >> 4], dim=-1)
    return out.reshape(*packed.shape[:-1], packed.shape[-1] * 2)


def dequant_v_affine_t(nib: torch.Tensor, scale: torch.Tensor, zero: torch.Tensor) -> torch.Tensor:
    return (nib.float() - zero.float().unsqueeze(-1)) * scale.float().unsqueeze(-1)


def dequant_v_sym_t(nib: torch.Tensor, scale: torch.Tensor, group: int = 32) -> torch.Tensor:
    shp = nib.shape
    g = (nib.float() - 8.0).reshape(*shp[:-1], shp[-1] // group, group)
    return (g * scale.float().unsqueeze(-1)).reshape(shp)


def quant_dequant_kv(k: torch.Tensor, v: torch.Tensor, layout: PageLayout) -> tuple[torch.Tensor, torch.Tensor]:
    """What the cache returns for fresh K/V: quantize then dequantize (fp32)."""
    fmt = layout.fmt
    kq, ks = quant_k_t(k, fmt.scale_dtype)
    kd = dequant_k_t(kq, ks)
    if fmt.v_mode == "affine_row":
        nib, vs, vz = quant_v_affine_t(v)
        vd = dequant_v_affine_t(nib, vs, vz)
    else:
        nib, vs = quant_v_sym_t(v, fmt.v_group)
        vd = dequant_v_sym_t(nib, vs, fmt.v_group)
    return kd, vd


def attention_ref(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    q_ends: torch.Tensor | list[int],
    gqa: int,
    quantize_q: bool = True,
    scale: float | None = None,
) -> torch.Tensor:
    """Causal GQA attention in fp32 for one sequence.

    ``q`` is ``[T, HQ, D]``, ``k``/``v`` ``[S, HKV, D]`` (already dequantized),
    ``q_ends[t]`` the number of keys query ``t`` sees. With ``quantize_q`` the
    query rows go through the int8 rule and K is re-quantized exactly (K from
    the cache is already on its int8 grid, so this reproduces the kernel's
    integer dot product).
    """
    T, HQ, Dh = q.shape
    S = k.shape[0]
    sc = (1.0 / math.sqrt(Dh)) if scale is None else scale
    ends = torch.as_tensor(q_ends, dtype=torch.int64)
    qf = q.float()
    if quantize_q:
        q8, qs = quant_k_t(qf, "float32")
        qf = q8.float() * qs.unsqueeze(-1)
    kh = k.float().repeat_interleave(gqa, dim=1)  # [S, HQ, D]
    vh = v.float().repeat_interleave(gqa, dim=1)
    scores = torch.einsum("thd,shd->hts", qf, kh) * sc
    keys = torch.arange(S).view(1, 1, S)
    mask = keys >= ends.view(1, T, 1)
    scores = scores.masked_fill(mask, float("-inf"))
    probs = torch.softmax(scores, dim=-1)
    probs = torch.nan_to_num(probs, nan=0.0)
    return torch.einsum("hts,shd->thd", probs, vh)


def sdpa_bf16_ref(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, gqa: int) -> torch.Tensor:
    """Unquantized bf16 causal (bottom-right) SDPA for one sequence, fp32 out."""
    T = q.shape[0]
    S = k.shape[0]
    qh = q.bfloat16().permute(1, 0, 2)
    kh = k.bfloat16().repeat_interleave(gqa, dim=1).permute(1, 0, 2)
    vh = v.bfloat16().repeat_interleave(gqa, dim=1).permute(1, 0, 2)
    ends = torch.arange(S - T + 1, S + 1)
    mask = torch.arange(S).view(1, S) < ends.view(T, 1)
    out = torch.nn.functional.scaled_dot_product_attention(qh.float(), kh.float(), vh.float(), attn_mask=mask)
    return out.permute(1, 0, 2).float()


def oracle_config(seed: int = 0, lens=(1024, 2048, 3072, 4096), hq: int = 24, hkv: int = 4, dim: int = 128):
    """The CPU decode-oracle workload: per-sequence bf16 q/k/v from N(0,1)."""
    gen = torch.Generator().manual_seed(seed)
    seqs = []
    for n in lens:
        k = torch.randn(n, hkv, dim, generator=gen).bfloat16()
        v = torch.randn(n, hkv, dim, generator=gen).bfloat16()
        q = torch.randn(1, hq, dim, generator=gen).bfloat16()
        seqs.append((q, k, v))
    return seqs


__all__ = [
    "quant_k", "dequant_k", "quant_v", "dequant_v", "causal_gqa", "deterministic_rows",
    "quant_k_t", "dequant_k_t", "quant_v_affine_t", "quant_v_sym_t", "pack_nibbles",
    "unpack_nibbles", "dequant_v_affine_t", "dequant_v_sym_t", "quant_dequant_kv",
    "attention_ref", "sdpa_bf16_ref", "oracle_config", "ref_layout",
]
