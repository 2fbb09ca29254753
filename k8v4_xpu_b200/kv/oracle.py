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
import random

import torch

from .layout import D, GQA, PageLayout, builtin_q_end, ref_layout

# ------------------------------------------------------------ scalar (lists)


def _rint(value: float) -> int:
    """Round half to even, like ``rintf`` / ``__float2int_rn``."""
    return int(round(value))


def _f32(x: float) -> float:
    return float(torch.tensor(x, dtype=torch.float32))


def quant_k(row: list[float]) -> tuple[list[int], float]:
    """Reference-format K row (fp32 scale)."""
    if len(row) != D:
        raise ValueError("K row must be %d" % D)
    q, s = quant_k_t(torch.tensor(row, dtype=torch.float32), "float32")
    return [int(v) for v in q.tolist()], float(s)


def dequant_k(packed: list[int], scale: float) -> list[float]:
    return [q * scale for q in packed]


def quant_v(row: list[float]) -> tuple[list[int], float, float]:
    """Reference-format V row: affine uint4, low nibble = even dim."""
    if len(row) != D:
        raise ValueError("V row must be %d" % D)
    nib, s, z = quant_v_affine_t(torch.tensor(row, dtype=torch.float32))
    packed = (nib[0::2] | (nib[1::2] << 4)).tolist()
    return [int(b) for b in packed], float(s), float(z)


def dequant_v(packed: list[int], scale: float, zero: float) -> list[float]:
    out: list[float] = []
    for byte in packed:
        out.append((float(byte & 0xF) - zero) * scale)
        out.append((float(byte >> 4) - zero) * scale)
    return out


def _softmax(scores: list[float]) -> list[float]:
    finite = [s for s in scores if s != float("-inf")]
    if not finite:
        return [0.0] * len(scores)
    peak = max(finite)
    exps = [0.0 if s == float("-inf") else math.exp(s - peak) for s in scores]
    total = sum(exps)
    if total == 0.0:
        return [0.0] * len(scores)
    inv = 1.0 / total
    return [e * inv for e in exps]


def causal_gqa(query, key, value, seq_len: int, q_len: int):
    """Quantized causal GQA over Python lists, reference format.

    ``query`` is ``[q_len][HQ][D]`` (the last ``q_len`` tokens), ``key`` and
    ``value`` are ``[seq_len][HKV][D]`` floats quantized here with the store
    rules. Behaviour of ``k8v4_v030/oracle.py:100-163``.
    """
    if len(query) != q_len:
        raise ValueError("query width")
    if len(key) < seq_len or len(value) < seq_len:
        raise ValueError("cache shorter than seq_len")
    if q_len == 0:
        return []
    kv_heads = len(key[0]) if key else len(query[0]) // GQA
    layout = PageLayout.for_heads(len(query[0]), kv_heads)
    hkv, hq = layout.hkv, layout.hq
    kq, vq = [], []
    for t in range(seq_len):
        k_heads, v_heads = [], []
        for h in range(hkv):
            k_heads.append(quant_k(key[t][h]))
            vp, vs, vz = quant_v(value[t][h])
            v_heads.append(dequant_v(vp, vs, vz))
        kq.append(k_heads)
        vq.append(v_heads)
    out = []
    inv_sqrt = 1.0 / math.sqrt(D)
    for q_tok in range(q_len):
        end = builtin_q_end(seq_len, q_len, q_tok)
        heads = []
        for h in range(hq):
            kv_head = h // GQA
            q_packed, q_scale = quant_k(query[q_tok][h])
            scores = []
            for t in range(seq_len):
                if t >= end:
                    scores.append(float("-inf"))
                    continue
                k_packed, k_scale = kq[t][kv_head]
                dot = sum(a * b for a, b in zip(q_packed, k_packed))
                scores.append(dot * q_scale * k_scale * inv_sqrt)
            probs = _softmax(scores)
            acc = [0.0] * D
            for t, prob in enumerate(probs):
                if prob == 0.0:
                    continue
                row = vq[t][kv_head]
                for d in range(D):
                    acc[d] += prob * row[d]
            heads.append(acc)
        out.append(heads)
    return out


def deterministic_rows(n: int, heads: int, seed: int, dim: int = D):
    rng = random.Random(seed)
    return [[[rng.uniform(-1.0, 1.0) for _d in range(dim)] for _h in range(heads)] for _ in range(n)]


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
