"""Python entry points of the sm_100a kernel library (``torch.ops.k8v4``).

The extension ``k8v4_xpu_b200._C`` is built in-tree by ``setup.py
build_ext --inplace`` (the reference loads its prebuilt ``libxe2_kv.so`` from
``XE2_KV_LIB`` the same way, ``k8v4_v030/ops_api.py:10-25``; ``K8V4_LIB`` is
the equivalent override here). On a machine with a CUDA device a missing or broken
extension raises instead of falling back to slower code: every op here runs
the CUDA kernel or fails loudly.
"""
from __future__ import annotations

import glob
import math
import os

import torch

_LOADED = False
_ERROR: str | None = None
# Kernel launches issued through this module (graph captures record deltas).
LAUNCHES = 0


def _count(n: int = 1) -> None:
    global LAUNCHES
    LAUNCHES += n


def load() -> bool:
    """Import the extension once. Returns False (and records why) on failure."""
    global _LOADED, _ERROR
    if _LOADED:
        return True
    try:
        path = _library_file()
        if path is None:
            raise ImportError("no built k8v4_xpu_b200/_C*.so")
        torch.ops.load_library(path)
        _ = torch.ops.k8v4.status
        _check_sources(path)
        _LOADED = True
        _ERROR = None
    except Exception as exc:  # pragma: no cover - depends on the build
        _ERROR = "%s: %s" % (type(exc).__name__, exc)
    return _LOADED


def _check_sources(path: str) -> None:
    """Refuse an in-tree library built from other sources than the csrc/
    tree beside the package (an explicit ``K8V4_LIB`` is taken as given)."""
    if os.environ.get("K8V4_LIB"):
        return
    from ..buildhash import source_hash
    csrc = os.path.join(os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))), "csrc")
    if not os.path.isdir(csrc):
        return  # an installed package without sources
    built, tree = str(torch.ops.k8v4.source_hash()), source_hash(csrc)
    if built != tree:
        raise ImportError("%s was built from other sources (%s) than csrc/ (%s); rebuild it" % (path, built, tree))


def require() -> None:
    """Raise if the kernel library is not usable."""
    if not load():
        raise RuntimeError(
            "k8v4 CUDA extension is not available (%s); build it with "
            "`python setup.py build_ext --inplace`" % _ERROR)


def available() -> bool:
    return load()


def _library_file() -> str | None:
    """The in-tree build, or ``K8V4_LIB`` (an explicit .so path) when set."""
    override = os.environ.get("K8V4_LIB")
    if override:
        return override if os.path.exists(override) else None
    pkg = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    found = sorted(glob.glob(os.path.join(pkg, "_C*.so")))
    return found[0] if found else None


def extension_path() -> str | None:
    """Path of the loaded in-tree kernel library."""
    if not load():
        return None
    return _library_file()


def status(clear: bool = True) -> int:
    """Device status word (0 = ok, 1 = a bounded wait timed out, ...)."""
    require()
    return int(torch.ops.k8v4.status(clear))


# ------------------------------------------------------------------ KV cache
FMT_REF, FMT_B200 = 0, 1


def kv_store(k: torch.Tensor, v: torch.Tensor, slots: torch.Tensor, cache: torch.Tensor, hkv: int,
             fmt: int = FMT_B200) -> None:
    require()
    torch.ops.k8v4.kv_store(fmt, k, v, slots, cache, hkv)
    _count()


def rope_store(qkv: torch.Tensor, cos_sin: torch.Tensor, positions: torch.Tensor, q_out: torch.Tensor,
               slots: torch.Tensor, cache: torch.Tensor, hq: int, hkv: int) -> None:
    """RoPE on the q / k heads of fused qkv rows, q written to ``q_out``, K and V
    quantized into their pages. ``qkv`` may be bf16 rows or the qkv GEMM's fp32
    split-K sums (then finished here and left zeroed for the next GEMM)."""
    require()
    torch.ops.k8v4.rope_store(qkv, cos_sin, positions, q_out, slots, cache, hq, hkv)
    _count()


def decode_ws_floats(nseq: int, heads: int, nsplit: int, max_q_len: int, gqa: int) -> int:
    require()
    return int(torch.ops.k8v4.decode_ws_floats(nseq, heads, nsplit, max_q_len, gqa))


def decode_attn(q, cu_q, seq_lens, block_table, cache, hkv, gqa, max_q_len, nsplit=1, out=None, ws=None,
                q_ends=None, head_offset=0, heads=None, sm_scale=None):
    """Split-K decode attention for every sequence of the batch in one launch."""
    require()
    heads = hkv if heads is None else heads
    if out is None:
        out = torch.empty_like(q)
    if sm_scale is None:
        sm_scale = 1.0 / math.sqrt(q.shape[-1])
    if nsplit > 1 and ws is None:
        ws = torch.empty(decode_ws_floats(seq_lens.numel(), heads, nsplit, max_q_len, gqa),
                         dtype=torch.float32, device=q.device)
    torch.ops.k8v4.decode_attn(q, cu_q, seq_lens, q_ends, block_table, cache, hkv, head_offset, heads, gqa,
                               max_q_len, nsplit, float(sm_scale), out, ws if nsplit > 1 else None)
    _count(2 if nsplit > 1 else 1)
    return out


def prefill_attn(q, cu_q, seq_lens, block_table, cache, hkv, gqa, max_q_len, out=None, head_offset=0,
                 heads=None, sm_scale=None):
    """Paged causal (bottom-right) attention of new tokens over their whole context."""
    require()
    heads = hkv if heads is None else heads
    if out is None:
        out = torch.empty_like(q)
    if sm_scale is None:
        sm_scale = 1.0 / math.sqrt(q.shape[-1])
    torch.ops.k8v4.prefill_attn(q, cu_q, seq_lens, block_table, cache, hkv, head_offset, heads, gqa, max_q_len,
                                float(sm_scale), out)
    _count()
    return out


# ---------------------------------------------------------------------- GEMM
W4A16, W4A8, W8A8 = 0, 1, 2


def wq_gemm(mode: int, w: torch.Tensor, wscale: torch.Tensor, x: torch.Tensor, xscale=None, residual=None,
            out=None, ws=None, split: int = 1, finish: bool = True) -> torch.Tensor:
    """Quantized-weight GEMM. With ``split > 1`` and ``finish=False`` the fp32
    partial sums stay in ``ws`` for a consumer that finishes them (the fused
    RMSNorm); ``out`` is then not written. A one-row W4A16 call given ``ws``
    runs as the decode GEMV (``takes_gemv``), which adds into ``ws`` even at
    ``split == 1``: a workspace passed here must be all zero, and it is left
    zero unless ``finish=False``."""
    require()
    n = w.shape[0] if mode == W8A8 else w.shape[1]
    if out is None:
        out = torch.empty((x.shape[0], n), dtype=torch.bfloat16, device=x.device)
    if split > 1 and ws is None:
        ws = torch.zeros((x.shape[0], n), dtype=torch.float32, device=x.device)
    if x.shape[0] == 0:
        return out
    torch.ops.k8v4.wq_gemm(mode, w, wscale, x, xscale, residual, out, ws, split, finish)
    if takes_gemv(mode, x.shape[0], ws):
        _count(2 if finish else 1)  # the GEMV, then the finish unless a consumer does it
    else:
        _count(2 if split > 1 and finish else 1)
    return out


GEMV_MAX_ROWS = 1


def takes_gemv(mode: int, rows: int, ws) -> bool:
    """Whether a GEMM call runs as the decode GEMV (``csrc/gemm/gemv_w4.cu``):
    W4A16 at one token row with an fp32 workspace, unless
    ``K8V4_DECODE_GEMV=0``. Mirrors the dispatch in ``csrc/bindings.cpp``."""
    if mode != W4A16 or not 1 <= rows <= GEMV_MAX_ROWS or ws is None:
        return False
    return os.environ.get("K8V4_DECODE_GEMV", "1")[:1] not in ("0", "n", "N", "f", "F")


# ------------------------------------------------------------------- fused
def wq_gemm_allreduce(mode: int, w, wscale, x, ws, ws_mc: int, flag_mc: int, xscale=None, split: int = 1,
                      gemv_local=None, gemv_ticket=None):
    """GEMM -> all-reduce: fp32 sums land in every rank's copy of ``ws`` (a
    symmetric buffer, multicast address ``ws_mc``); the call then signals the
    multicast counter ``flag_mc`` (``wq_gemm_ctas`` times per rank). A
    one-row W4A16 call runs as the decode GEMV, whose partial sums first meet
    in ``gemv_local`` (fp32, zero, left zero) and whose last CTA, picked by
    ``gemv_ticket`` (int32, zero, left zero), sends the rows. Returns ``ws``."""
    require()
    if x.shape[0] == 0:
        return ws
    torch.ops.k8v4.wq_gemm_allreduce(mode, w, wscale, x, xscale, ws, int(ws_mc), int(flag_mc), int(split),
                                     gemv_local, gemv_ticket)
    _count()
    return ws


def wq_gemm_sp(mode: int, w, wscale, x, world: int, rank: int, tile0, xscale=None, out=None, ag_flag: int = 0,
               ag_target=(), rs_dst=(), rs_sig=()):
    """Sequence-parallel prefill GEMM over 128-row token tiles owned by ranks
    (``tile0[o]`` .. ``tile0[o + 1]`` for rank ``o``). With ``ag_flag`` (the
    address of this rank's per-owner row counters) ``x`` is this rank's copy of
    the all-gathered rows and each CTA waits for its tile's owner; the output
    goes to ``out``. With ``rs_dst`` / ``rs_sig`` (peer addresses per owner)
    the output goes as bf16 partial rows into the owners' slots instead."""
    require()
    if ag_flag == 0 and not rs_dst:
        raise ValueError("wq_gemm_sp needs a gather wait or a scatter")
    n = w.shape[1]
    if not rs_dst and out is None:
        out = torch.empty((x.shape[0], n), dtype=torch.bfloat16, device=x.device)
    torch.ops.k8v4.wq_gemm_sp(mode, w, wscale, x, xscale, out, int(world), int(rank), [int(t) for t in tile0],
                              int(ag_flag), [int(t) for t in ag_target], [int(a) for a in rs_dst],
                              [int(a) for a in rs_sig])
    _count()
    return out


def rmsnorm_sp(residual, w, rows: int, eps: float, slots=None, world: int = 1, slot_stride: int = 0, x_local=None,
               init_residual: bool = False, rs_flag: int = 0, rs_target: int = 0, y: int = 0, yq: int = 0,
               ys: int = 0, row0: int = 0, mc: bool = False, ag_sig: int = 0) -> None:
    """Sequence-parallel norm of ``rows`` local rows: slots summed (after the
    reduce-scatter signals) or ``x_local``, plus the residual, normalized, and
    pushed to every rank through multicast addresses (``mc``) or written to
    local addresses ``y`` / ``yq`` + ``ys``."""
    require()
    if rows <= 0:
        return
    torch.ops.k8v4.rmsnorm_sp(slots, int(world), int(slot_stride), x_local, residual, bool(init_residual), w,
                              int(rows), float(eps), int(rs_flag), int(rs_target), int(y), int(yq), int(ys),
                              int(row0), bool(mc), int(ag_sig))
    _count()


def wq_gemm_ctas(mode: int, M: int, N: int, K: int, split: int = 1) -> int:
    require()
    return int(torch.ops.k8v4.wq_gemm_ctas(mode, M, N, K, split))


def rmsnorm(x, w, eps=1e-6, residual=None, out=None, quant=False, sync=None):
    """RMSNorm (optionally residual-add first); returns y, or (q, scale) with quant.

    ``x`` may be the fp32 split-K accumulator of the preceding GEMM: it is
    consumed (and zeroed) here, finishing that GEMM inside the norm. With
    ``sync = (flag, state, expected)`` x is this rank's copy of a GEMM ->
    all-reduce buffer and the norm first waits for every rank's signals.
    """
    require()
    rows = x.numel() // x.shape[-1]
    sf, ss, se = sync if sync is not None else (None, None, 0)
    if quant:
        q = torch.empty(x.shape, dtype=torch.int8, device=x.device)
        s = torch.empty(rows, dtype=torch.float32, device=x.device)
        torch.ops.k8v4.rmsnorm(x, residual, w, out, q, s, eps, sf, ss, int(se))
        _count()
        return (out, q, s) if out is not None else (q, s)
    if out is None:
        out = torch.empty(x.shape, dtype=torch.bfloat16, device=x.device)
    torch.ops.k8v4.rmsnorm(x, residual, w, out, None, None, eps, sf, ss, int(se))
    _count()
    return out


def int8_dequant(q, scale, out):
    """INT8 island weights ``q`` [N, K] x per-row ``scale`` [N] -> bf16 into ``out`` (>= N*K elements)."""
    require()
    torch.ops.k8v4.int8_dequant(q, scale, out)
    _count()
    return out[: q.numel()].view(q.shape)


def silu_mul(gu, out=None, quant=False):
    """silu(gate) * up of ``gu = [gate | up]`` (bf16, or int8 + per-row scale
    with ``quant``). ``gu`` may be the fp32 sums a decode GEMV left in the
    split-K workspace (bf16 output only): they are consumed and zeroed."""
    require()
    rows, inter = gu.shape[0], gu.shape[1] // 2
    if gu.dtype == torch.float32:
        if quant:
            raise ValueError("silu_mul of fp32 sums writes bf16 only")
        if out is None:
            out = torch.empty((rows, inter), dtype=torch.bfloat16, device=gu.device)
        torch.ops.k8v4.silu_mul_f32(gu, out)
        _count()
        return out
    if quant:
        q = torch.empty((rows, inter), dtype=torch.int8, device=gu.device)
        s = torch.empty(rows, dtype=torch.float32, device=gu.device)
        torch.ops.k8v4.silu_mul(gu, out, q, s)
        _count()
        return q, s
    if out is None:
        out = torch.empty((rows, inter), dtype=torch.bfloat16, device=gu.device)
    torch.ops.k8v4.silu_mul(gu, out, None, None)
    _count()
    return out


def quant_rows(x):
    require()
    q = torch.empty(x.shape, dtype=torch.int8, device=x.device)
    s = torch.empty(x.numel() // x.shape[-1], dtype=torch.float32, device=x.device)
    torch.ops.k8v4.quant_rows(x, q, s)
    _count()
    return q, s


def embed_int8(ids, codes, scales, start=0, out=None):
    require()
    if out is None:
        out = torch.empty((ids.numel(), codes.shape[1]), dtype=torch.bfloat16, device=codes.device)
    torch.ops.k8v4.embed_int8(ids, codes, scales, out, int(start))
    _count()
    return out


def argmax(logits, offset=0):
    require()
    v = torch.empty(logits.shape[0], dtype=torch.float32, device=logits.device)
    i = torch.empty(logits.shape[0], dtype=torch.int64, device=logits.device)
    torch.ops.k8v4.argmax(logits, int(offset), v, i)
    _count()
    return v, i


def gather_dequant(cache, block_table, hkv: int, head: int, seq_len: int, dtype=torch.float32):
    """Dense ``[seq_len, 128]`` K and V of one KV head from its pages (b200 format)."""
    require()
    k = torch.empty((seq_len, 128), dtype=dtype, device=cache.device)
    v = torch.empty((seq_len, 128), dtype=dtype, device=cache.device)
    torch.ops.k8v4.gather_dequant(cache, block_table.to(torch.int32).contiguous(), hkv, head, seq_len, k, v)
    _count()
    return k, v


def prefill_attn_cp(q, cu_q, seq_lens, block_table, caches, hkv, gqa, max_q_len, q_pos=None, out=None,
                    head_offset=0, heads=None, sm_scale=None):
    """Paged causal prefill reading pages from several KV caches (context
    parallelism): entry ``(source << 24) | page`` of the block table addresses
    ``caches[source]``; ``q_pos`` gives each query token's global position."""
    require()
    heads = hkv if heads is None else heads
    if out is None:
        out = torch.empty_like(q)
    scale = (1.0 / math.sqrt(q.shape[-1])) if sm_scale is None else sm_scale
    torch.ops.k8v4.prefill_attn_cp(q, cu_q, seq_lens, block_table, list(caches), q_pos, hkv, head_offset, heads, gqa,
                                   max_q_len, float(scale), out)
    _count()
    return out


def decode_combine_ranks(ws_all, rank_floats: int, cu_q, nrank: int, nsplit: int, heads: int, gqa: int,
                         max_q_len: int, out, head_offset: int = 0, sync=None):
    """Merge the split-K partials of every context-parallel rank into ``out``.

    ``sync`` = (counter, state, expected) when ``ws_all`` is this rank's copy
    of the gather buffer that :func:`decode_attn_push` fills: the kernel first
    waits until the counter holds ``expected`` more signals (bounded)."""
    require()
    flag, state, expected = sync if sync is not None else (None, None, 0)
    torch.ops.k8v4.decode_combine_ranks(ws_all, int(rank_floats), cu_q, nrank, nsplit, heads, head_offset, gqa,
                                        max_q_len, out, flag, state, int(expected))
    _count()
    return out


def decode_attn_push(q, cu_q, seq_lens, block_table, cache, hkv, gqa, max_q_len, nsplit, slot_mc: int,
                     flag_mc: int, q_ends=None, head_offset=0, heads=None, sm_scale=None):
    """Split-K decode attention whose partials go straight into every rank's
    copy of this rank's gather slot (``slot_mc``: its multicast address),
    then one signal per CTA on the multicast counter ``flag_mc``."""
    require()
    heads = hkv if heads is None else heads
    if sm_scale is None:
        sm_scale = 1.0 / math.sqrt(q.shape[-1])
    torch.ops.k8v4.decode_attn_push(q, cu_q, seq_lens, q_ends, block_table, cache, hkv, head_offset, heads, gqa,
                                    max_q_len, nsplit, float(sm_scale), int(slot_mc), int(flag_mc))
    _count()
    return q


def decode_push_ctas(nseq: int, heads: int, nsplit: int) -> int:
    """Signals one :func:`decode_attn_push` launch sends (its CTAs)."""
    return int(nseq) * int(heads) * int(nsplit)


def enable_peer_access(peer_device: int) -> bool:
    """Grant the current device access to ``peer_device``'s memory."""
    require()
    return bool(torch.ops.k8v4.enable_peer_access(int(peer_device)))
