"""Quantized linear layers and the W4A8 / W4A16 path policy.

Every linear of the decoder stores GPTQ INT4 (group 128) weights. The path
choice follows the reference's MLP-only rule (``k8v4_v030/w4a8_prefill.py:
19,160-176,237-252``): a linear whose name contains ``.mlp.`` runs W4A8
(int8 activations with a per-token scale) when the call has more than
``SMALL_M_MAX`` rows; everything else (attention projections at any M and
every linear at decode sizes) runs W4A16. Both are the same tcgen05 kernel
family (``csrc/gemm/wq_gemm.cu``); the choice is made per call from the
runtime row count, so one captured decode graph and an eager prefill chunk
can each take the right path.
"""
from __future__ import annotations

import os

import torch

from .. import ops

SMALL_M_MAX = 128
NUM_SMS = 148


def w4a8_enabled() -> bool:
    """``K8V4_PREFILL_GEMM`` = ``w4a8`` (default) or ``w4a16`` (MLP keeps W4A16).

    The default is the reference deployment's (``k8v4_v030/launch.sh:160``
    sets ``w4a8``; the module's own fallback is ``w4a16``,
    ``k8v4_v030/w4a8_prefill.py:385``)."""
    mode = os.environ.get("K8V4_PREFILL_GEMM", "w4a8").strip().lower()
    if mode not in ("w4a8", "w4a16"):
        raise ValueError("K8V4_PREFILL_GEMM must be w4a8 or w4a16, got %r" % mode)
    return mode == "w4a8"


def uses_w4a8(name: str, rows: int, enabled: bool = True) -> bool:
    """The reference's runtime gate: MLP linears, rows > SMALL_M_MAX."""
    return enabled and ".mlp." in name and rows > SMALL_M_MAX


_NOTED: set = set()


def note_gemm_branch(name: str, rows: int, branch: str, env=None) -> None:
    """``K8V4_GEMM_DIAGNOSTICS=1``: log which GEMM path a linear took, once
    per (linear, path) (the reference's switch, ``w4a8_prefill.py:227,240-244``)."""
    if (os.environ if env is None else env).get("K8V4_GEMM_DIAGNOSTICS", "0") in ("", "0"):
        return
    key = (name, branch)
    if key in _NOTED:
        return
    _NOTED.add(key)
    import logging
    logging.getLogger("k8v4").info("gemm %s: %s (first at %d rows)", name, branch, rows)


def split_for(rows: int, n: int, k: int, sms: int = NUM_SMS) -> int:
    """Split-K factor that fills the GPU for skinny (decode) GEMMs."""
    if rows > 64:
        return 1
    tiles = (n + 127) // 128
    if tiles >= sms:
        return 1
    groups = k // 128
    split = max(1, min(sms // tiles, groups // 4 if groups >= 8 else 1))
    return split


class Int4Linear:
    """GPTQ INT4 weights ``qweight`` [K/8, N] int32 + ``scales`` [K/128, N] fp16."""

    supports_w4a8 = True  # takes int8 activations on the MLP prefill path

    def __init__(self, name: str, qweight: torch.Tensor, scales: torch.Tensor):
        if qweight.dim() != 2 or scales.dim() != 2:
            raise ValueError("qweight / scales must be 2D")
        self.name = name
        self.qweight = qweight
        self.scales = scales
        self.in_features = qweight.shape[0] * 8
        self.out_features = qweight.shape[1]

    def split(self, rows: int, ws) -> int:
        return split_for(rows, self.out_features, self.in_features) if ws is not None else 1

    def __call__(self, x: torch.Tensor | None = None, xq: torch.Tensor | None = None,
                 xs: torch.Tensor | None = None, out: torch.Tensor | None = None,
                 ws: torch.Tensor | None = None, split: int | None = None, defer: bool = False) -> torch.Tensor:
        """Run the GEMM. With ``defer`` and a split-K launch, returns the fp32
        partial-sum view of ``ws`` (rows x out_features) for a fused consumer."""
        if xq is not None:
            return ops.wq_gemm(ops.W4A8, self.qweight, self.scales, xq, xscale=xs, out=out)
        rows = x.shape[0]
        if split is None:
            split = self.split(rows, ws)
        if defer and (split > 1 or ops.takes_gemv(ops.W4A16, rows, ws)):
            ops.wq_gemm(ops.W4A16, self.qweight, self.scales, x, out=out, ws=ws, split=split, finish=False)
            return ws[: rows * self.out_features].view(rows, self.out_features)
        return ops.wq_gemm(ops.W4A16, self.qweight, self.scales, x, out=out, ws=ws, split=split)

    def reference(self, x: torch.Tensor) -> torch.Tensor:
        from ..models.gptq import dequant_int4
        return x.float() @ dequant_int4(self.qweight, self.scales)

    def dense_t(self) -> torch.Tensor:
        """The dequantized weight [K, N] in fp32 on the CPU (torch reference paths)."""
        from ..models.gptq import dequant_int4
        return dequant_int4(self.qweight.cpu(), self.scales.cpu())


class Int8RowLinear:
    """Per-row INT8 weights ``[N, K]`` + fp16 scales ``[N]`` (the lm_head).

    The GEMM tiles output features by 128, so the rows are zero-padded to a
    multiple of 128 (a vocab shard under TP, e.g. 151936 / 2 = 75968, is not);
    the call returns a view over the real rows.
    """

    def __init__(self, name: str, weight: torch.Tensor, scale: torch.Tensor):
        self.name = name
        n, k = weight.shape
        pad = (-n) % 128
        if pad:
            weight = torch.cat([weight, weight.new_zeros(pad, k)])
            scale = torch.cat([scale.reshape(-1), scale.new_zeros(pad)])
        self.weight = weight.contiguous()
        self.scale = scale.reshape(-1).contiguous()
        self.out_features, self.in_features = n, k

    def __call__(self, xq: torch.Tensor, xs: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        y = ops.wq_gemm(ops.W8A8, self.weight, self.scale, xq, xscale=xs, out=out)
        return y if y.shape[1] == self.out_features else y[:, : self.out_features]


# ------------------------------------------------------------------ INT8 islands
def island_suffixes(env=None) -> tuple[str, ...]:
    """Module-name suffixes listed in ``K8V4_INT8_ISLANDS`` (comma separated),
    the reference's switch (``k8v4_v030/int8_island.py:50-53``)."""
    raw = (os.environ if env is None else env).get("K8V4_INT8_ISLANDS", "")
    return tuple(x.strip() for x in raw.split(",") if x.strip())


def is_island(name: str, suffixes: tuple[str, ...]) -> bool:
    return any(name.endswith(suf) for suf in suffixes)


_SCRATCH: dict = {}


def _island_scratch(numel: int, device) -> torch.Tensor:
    """One bf16 buffer per device for the dequantized island weight (grows,
    never shrinks, so a captured graph keeps its address)."""
    key = str(device)
    buf = _SCRATCH.get(key)
    if buf is None or buf.numel() < numel:
        buf = torch.empty(numel, dtype=torch.bfloat16, device=device)
        _SCRATCH[key] = buf
    return buf


class Int8IslandLinear:
    """A dense linear kept resident as per-output-row symmetric int8 weights
    ``q`` [N, K] with bf16 scales [N] (the reference's INT8 island,
    ``k8v4_v030/int8_island.py:60-130``: ``s = max(amax / 127, 1e-12)``,
    ``q = round(w / s)`` clamped to +-127). The product is W8A16 on the
    in-tree tcgen05 int8 GEMM: the bf16 activations are split into two int8
    limbs per row (x ~= s1 q1 + s2 q2, the second quantizing the residual of
    the first, ~14 bits against the row's amax) and the W8A8 GEMM runs once
    per limb, both adding fp32 sums into one accumulator that the second
    call finishes to bf16. The weight bytes are read twice, against five per
    weight when dequantizing into a bf16 scratch for a library GEMM (kept for
    shapes the GEMM does not tile: K not a multiple of 128). Islands halve
    the weight memory of the dense layers they replace; they are not a hot
    path.
    """

    supports_w4a8 = False

    def __init__(self, name: str, q: torch.Tensor, scale: torch.Tensor):
        if q.dtype != torch.int8 or q.dim() != 2:
            raise ValueError("island weights must be int8 [N, K]")
        self.name = name
        self.q = q.contiguous()
        self.scale = scale.reshape(-1).to(torch.bfloat16).contiguous()
        self.out_features, self.in_features = q.shape
        # the int8 GEMM's operands: rows padded to its 128-row tile, fp16
        # scales (exact for bf16 scales inside the fp16 normal range)
        self._gemm = None
        n, k = self.q.shape
        s32 = self.scale.float().abs()
        if k % 128 == 0 and bool(((s32 == 0) | ((s32 >= 6.2e-5) & (s32 <= 6.5e4))).all()):
            pad = (-n) % 128
            qp = torch.cat([self.q, self.q.new_zeros(pad, k)]) if pad else self.q
            sp = torch.cat([self.scale, self.scale.new_zeros(pad)]) if pad else self.scale
            self._gemm = (qp.contiguous(), sp.to(torch.float16).contiguous())

    @staticmethod
    def quantize(w: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        """Dense [N, K] -> (int8 [N, K], bf16 [N])."""
        w = w.float()
        s = (w.abs().amax(dim=1, keepdim=True) / 127.0).clamp_min(1e-12)
        q = torch.round(w / s).clamp_(-127, 127).to(torch.int8)
        return q, s.reshape(-1).to(torch.bfloat16)

    @classmethod
    def from_dense(cls, name: str, w: torch.Tensor, device=None) -> "Int8IslandLinear":
        q, s = cls.quantize(w)
        return cls(name, q.to(device) if device is not None else q, s.to(device) if device is not None else s)

    def __call__(self, x: torch.Tensor | None = None, xq=None, xs=None, out: torch.Tensor | None = None,
                 ws=None, split=None, defer: bool = False) -> torch.Tensor:
        if x is None:
            raise ValueError("%s: INT8 islands take bf16 activations" % self.name)
        if self._gemm is not None and x.is_cuda and x.dim() == 2 and x.shape[0] > 0:
            y = self._two_limb_gemm(x)
        else:
            w = ops.int8_dequant(self.q, self.scale, _island_scratch(self.q.numel(), self.q.device))
            y = torch.matmul(x, w.t())
        if out is not None:
            out.copy_(y)
            return out
        return y

    def _two_limb_gemm(self, x: torch.Tensor) -> torch.Tensor:
        qp, sp = self._gemm
        rows = x.shape[0]
        q1, s1 = ops.quant_rows(x.contiguous())
        resid = (x.float() - q1.float() * s1.view(-1, 1)).to(torch.bfloat16)
        q2, s2 = ops.quant_rows(resid)
        ws = torch.zeros(rows * qp.shape[0], dtype=torch.float32, device=x.device)
        ops.wq_gemm(ops.W8A8, qp, sp, q1, xscale=s1, ws=ws, split=2, finish=False)
        y = ops.wq_gemm(ops.W8A8, qp, sp, q2, xscale=s2, ws=ws, split=2)
        return y if y.shape[1] == self.out_features else y[:, : self.out_features]

    def reference(self, x: torch.Tensor) -> torch.Tensor:
        return x.float() @ (self.q.float() * self.scale.float()[:, None]).t()

    def dense_t(self) -> torch.Tensor:
        """The dequantized weight [K, N] in fp32 on the CPU (torch reference paths)."""
        return (self.q.float().cpu() * self.scale.float().cpu()[:, None]).t()
