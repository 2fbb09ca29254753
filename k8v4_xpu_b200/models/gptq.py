"""GPTQ INT4 (group 128, symmetric) and INT8 per-row weight formats.

Checkpoint format (the reference's bake, ``tools/bake_gptq_resume.py:51-75``):

* ``qweight`` int32 ``[K/8, N]``: eight consecutive K codes of one output
  column per word, low nibble first; code = q + 8 with q in [-8, 7];
* ``scales`` fp16 ``[K/128, N]``: ``amax(|w|) / 7`` over each 128-row group;
* ``qzeros`` int32 ``[K/128, N/8]`` all ``0x77777777``; ``g_idx = k // 128``;
  ``desc_act`` false.

INT8 per-row (embedding side file and lm_head, ``tools/assemble_swift_bake.py
:100-106``): codes int8 ``[V, H]`` = ``round(w / s)`` clamped to
[-128, 127] with ``s = amax(|row|) / 127`` stored fp16 ``[V, 1]``.

This module holds the CPU/torch reference of both formats: quantizers (round
to nearest; the Hessian-based GPTQ solve of the offline bake is in
``k8v4_xpu_b200.tools.bake``), packers, unpackers and dequantized matmuls the
CUDA GEMMs are tested against.
"""
from __future__ import annotations

import torch

GROUP = 128
QZERO_WORD = 0x77777777


def quantize_int4_rtn(w_kn: torch.Tensor, group: int = GROUP) -> tuple[torch.Tensor, torch.Tensor]:
    """Round-to-nearest symmetric int4 of ``w`` laid out ``[K, N]``.

    Returns (codes uint8 [K, N] in 0..15, scales fp32 [K/group, N]).
    """
    K, N = w_kn.shape
    if K % group:
        raise ValueError("K must be a multiple of %d" % group)
    w = w_kn.float().reshape(K // group, group, N)
    s = w.abs().amax(dim=1).clamp_min(1e-9) / 7.0
    s16 = s.half().float()  # quantize against the stored fp16 scale
    q = torch.clamp(torch.round(w / s16.unsqueeze(1)), -8, 7)
    return (q + 8).to(torch.uint8).reshape(K, N), s16


def pack_int4(codes_kn: torch.Tensor, scales: torch.Tensor) -> dict[str, torch.Tensor]:
    """GPTQ tensors from codes ``[K, N]`` (0..15) and per-group scales."""
    K, N = codes_kn.shape
    c = codes_kn.to(torch.int64).reshape(K // 8, 8, N)
    sh = (torch.arange(8, dtype=torch.int64) * 4).view(1, 8, 1).to(c.device)
    qweight = (c << sh).sum(1).to(torch.int64)
    qweight = torch.where(qweight >= 2**31, qweight - 2**32, qweight).to(torch.int32)
    groups = K // GROUP
    return {
        "qweight": qweight.contiguous(),
        "scales": scales.half().contiguous(),
        "qzeros": torch.full((groups, max(1, N // 8)), QZERO_WORD, dtype=torch.int32, device=c.device),
        "g_idx": (torch.arange(K, dtype=torch.int32, device=c.device) // GROUP),
    }


def unpack_int4(qweight: torch.Tensor) -> torch.Tensor:
    """codes uint8 ``[K, N]`` from ``qweight`` ``[K/8, N]``."""
    K8, N = qweight.shape
    sh = (torch.arange(8, dtype=torch.int32, device=qweight.device) * 4).view(1, 8, 1)
    return ((qweight.unsqueeze(1) >> sh) & 0xF).reshape(K8 * 8, N).to(torch.uint8)


def dequant_int4(qweight: torch.Tensor, scales: torch.Tensor, group: int = GROUP) -> torch.Tensor:
    """fp32 ``[K, N]`` = (code - 8) * scale."""
    codes = unpack_int4(qweight).float() - 8.0
    K, N = codes.shape
    return (codes.reshape(K // group, group, N) * scales.float().unsqueeze(1)).reshape(K, N)


def quantize_int8_rows(w: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Per-row int8: (codes int8 [V, H], scale fp16 [V, 1])."""
    w = w.float()
    s = (w.abs().amax(dim=1, keepdim=True) / 127.0).clamp_min(1e-12).half()
    q = torch.clamp(torch.round(w / s.float()), -128, 127).to(torch.int8)
    return q, s


def w4a16_ref(x: torch.Tensor, qweight: torch.Tensor, scales: torch.Tensor) -> torch.Tensor:
    """fp32 reference of the W4A16 GEMM: x (bf16) @ dequant(W)."""
    return x.float() @ dequant_int4(qweight, scales)


def w4a8_ref(xq: torch.Tensor, xs: torch.Tensor, qweight: torch.Tensor, scales: torch.Tensor) -> torch.Tensor:
    """fp32 reference of the W4A8 GEMM: per-group integer dots, fp32 group scales."""
    codes = unpack_int4(qweight).to(torch.int64) - 8  # [K, N]
    K, N = codes.shape
    xi = xq.to(torch.int64)
    acc = torch.zeros((xq.shape[0], N), dtype=torch.float64)
    for g in range(K // GROUP):
        part = xi[:, g * GROUP:(g + 1) * GROUP] @ codes[g * GROUP:(g + 1) * GROUP]
        acc += part.double() * scales[g].double()
    return (acc * xs.double().view(-1, 1)).float()


def w8a8_ref(xq: torch.Tensor, xs: torch.Tensor, wq: torch.Tensor, ws: torch.Tensor) -> torch.Tensor:
    acc = xq.to(torch.int64) @ wq.to(torch.int64).t()
    return (acc.double() * ws.double().view(1, -1) * xs.double().view(-1, 1)).float()


def quant_act_rows(x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Per-token int8 activations, the reference's rule (``w4a8_prefill.py:192-203``):
    scale = max(amax/127, 1e-5), codes = clamp(round(x/scale), -127, 127)."""
    xf = x.float()
    s = torch.clamp(xf.abs().amax(dim=-1) / 127.0, min=1e-5)
    inv = 1.0 / s
    q = torch.clamp(torch.round(xf * inv.unsqueeze(-1)), -127, 127).to(torch.int8)
    return q, s
