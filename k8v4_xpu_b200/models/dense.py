"""The dense K8/V4 decoder: weights, random init, and the forward pass.

Per layer (one rank of a TP group):

    residual, h = rmsnorm(x + residual)            fused add + norm
    qkv         = h @ Wqkv                         W4A16 (tcgen05); decode: fp32 split-K sums
    q, K/V      = rope_store(qkv)                  (finish split-K +) RoPE + K8/V4 page write
    a           = paged attention(q, pages)        decode: split-K; prefill: causal tiles
    x           = a @ Wo                           W4A16, then TP all-reduce
    residual, h = rmsnorm(x + residual)            (+ int8 quant when W4A8 runs)
    gu          = h @ Wgate_up                     W4A8 above 128 rows, else W4A16
    act         = silu(gate) * up                  (+ int8 quant)
    x           = act @ Wdown                      then TP all-reduce

The embedding is the INT8 side-file lookup (vocab sharded under TP), the
lm_head is INT8 per-row with int8 activations, sampling is a per-rank argmax
reduced across ranks. Attention metadata (slots, block tables, lengths) comes
in a :class:`StepInputs`. A layer listed in ``skip_kv`` (set by the engine
from ``kv_cache_dtype_skip_layers``) keeps its KV in plain fp8 / bf16 pages
and runs RoPE, store and attention through ``kv.skip_layers`` instead of
``rope_store`` and the K8/V4 attention kernels.

Reference counterparts: the K8/V4 attention backend
(``k8v4_v030/backend.py:79-486``), the MLP-only W4A8 prefill hook
(``k8v4_v030/w4a8_prefill.py:146-157,382-392``) and the INT8 embedding
runtime (``k8v4_v030/embed_int8_runtime.py:11-56``); the rest of the decoder
is stock vLLM there.
"""
from __future__ import annotations

import dataclasses
import math

import torch

from .. import ops
from ..kv import skip_layers
from ..kv.layout import PageLayout, b200_layout
from ..layers.linear import Int4Linear, Int8RowLinear, note_gemm_branch, uses_w4a8, w4a8_enabled
from ..obs.attn_time import attention_span
from ..obs.stage_profile import stage
from . import gptq
from .config import ModelConfig, TPShape


@dataclasses.dataclass
class StepInputs:
    """Device tensors describing one forward over a packed token batch."""

    input_ids: torch.Tensor      # [T] int64
    positions: torch.Tensor      # [T] int64
    slots: torch.Tensor          # [T] int64 KV slot of each token
    cu_q: torch.Tensor           # [B+1] int32
    seq_lens: torch.Tensor       # [B] int32 (context incl. these tokens)
    block_table: torch.Tensor    # [B, W] int32
    logit_rows: torch.Tensor     # [B'] int64 rows of the batch whose logits are needed
    max_q_len: int
    is_decode: bool              # every sequence has q_len <= the decode tile
    q_ends: torch.Tensor | None = None  # [T] int32 per-token visible end (MTP trees)
    nsplit: int = 1              # decode split-K factor
    # context parallelism: global positions of this rank's rows (prefill), and
    # this rank's own pages of every sequence with the keys they hold (decode)
    q_pos: torch.Tensor | None = None        # [T] int32
    cp_local_bt: torch.Tensor | None = None  # [B, W] int32
    cp_local_lens: torch.Tensor | None = None  # [B] int32


@dataclasses.dataclass
class LayerWeights:
    input_norm: torch.Tensor
    post_norm: torch.Tensor
    qkv: Int4Linear
    o: Int4Linear
    gate_up: Int4Linear
    down: Int4Linear


@dataclasses.dataclass
class MTPWeights:
    enorm: torch.Tensor
    hnorm: torch.Tensor
    norm: torch.Tensor
    eh_proj: Int4Linear
    layer: LayerWeights


def rope_table(max_pos: int, head_dim: int, theta: float, device) -> torch.Tensor:
    """fp32 ``[max_pos, head_dim]``: cos of the half-dim frequencies then sin."""
    inv = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.float64) / head_dim))
    pos = torch.arange(max_pos, dtype=torch.float64)
    ang = pos.view(-1, 1) * inv.view(1, -1)
    return torch.cat([ang.cos(), ang.sin()], dim=1).float().to(device)


def _rand_int4(k: int, n: int, gen: torch.Generator, device, std: float = 0.02):
    w = torch.randn(k, n, generator=gen, device=device) * std
    codes, scales = gptq.quantize_int4_rtn(w)
    t = gptq.pack_int4(codes, scales)
    return t["qweight"], t["scales"]


class DenseModel:
    """One TP rank of the dense decoder (weights resident on ``device``)."""

    def __init__(self, cfg: ModelConfig, tp: int = 1, rank: int = 0, device="cuda", comm=None):
        self.cfg = cfg
        self.tp = tp
        self.rank = rank
        self.device = torch.device(device)
        self.shape: TPShape = cfg.tp_shard(tp)
        self.comm = comm
        self.layout: PageLayout = b200_layout(self.shape.hkv_local, self.shape.gqa_local)
        self.layers: list[LayerWeights] = []
        self.embed_codes = self.embed_scales = None
        self.final_norm = None
        self.lm_head: Int8RowLinear | None = None
        self.vocab_start = rank * self.shape.vocab_local
        self.rope = None
        self.w4a8 = w4a8_enabled()
        self.mtp = None
        # layer index (the MTP layer: len(layers)) -> plain fp8 / bf16 cache layout
        self.skip_kv: dict[int, skip_layers.SkipLayout] = {}
        self.fused_ar = None  # parallel.fused_ar.FusedAllReduce when TP runs the fused path
        self.sp = None        # parallel.seq_parallel.SeqParallel: fused reduce-scatter / all-gather prefill
        self.cp = None        # parallel.cp.CPGroup under context parallelism

    # ------------------------------------------------------------- weights
    def random_init(self, seed: int = 0, layers: int | None = None) -> "DenseModel":
        """Random-init weights of the architecture, quantized on the device.

        Every rank draws the *full* matrices from the same seed and keeps its
        shard, so TP ranks hold a consistent model.
        """
        cfg, sh = self.cfg, self.shape
        dev = self.device
        gen = torch.Generator(device=dev).manual_seed(seed)
        H, D = cfg.hidden, cfg.head_dim
        n_layers = cfg.num_layers if layers is None else layers
        self.layers = []
        for li in range(n_layers):
            qkv_q, qkv_s = self._shard_qkv(*_rand_int4(H, cfg.q_size + 2 * cfg.kv_size, gen, dev))
            o_q, o_s = _rand_int4(cfg.q_size, H, gen, dev)
            o_q, o_s = self._shard_rows(o_q, o_s, sh.hq_local * D)
            gu_q, gu_s = _rand_int4(H, 2 * cfg.intermediate, gen, dev)
            gu_q, gu_s = self._shard_gate_up(gu_q, gu_s)
            dn_q, dn_s = _rand_int4(cfg.intermediate, H, gen, dev)
            dn_q, dn_s = self._shard_rows(dn_q, dn_s, sh.inter_local)
            pre = "model.layers.%d." % li
            self.layers.append(LayerWeights(
                input_norm=(1.0 + 0.02 * torch.randn(H, generator=gen, device=dev)).bfloat16(),
                post_norm=(1.0 + 0.02 * torch.randn(H, generator=gen, device=dev)).bfloat16(),
                qkv=Int4Linear(pre + "self_attn.qkv_proj", qkv_q, qkv_s),
                o=Int4Linear(pre + "self_attn.o_proj", o_q, o_s),
                gate_up=Int4Linear(pre + "mlp.gate_up_proj", gu_q, gu_s),
                down=Int4Linear(pre + "mlp.down_proj", dn_q, dn_s),
            ))
        V = cfg.vocab
        v0, v1 = self.vocab_start, self.vocab_start + sh.vocab_local
        emb = torch.randn(V, H, generator=gen, device=dev) * 0.02
        codes, scales = gptq.quantize_int8_rows(emb[v0:v1])
        self.embed_codes, self.embed_scales = codes.contiguous(), scales.view(-1).contiguous()
        del emb
        head = torch.randn(V, H, generator=gen, device=dev) * 0.02
        hq, hs = gptq.quantize_int8_rows(head[v0:v1])
        self.lm_head = Int8RowLinear("lm_head", hq.contiguous(), hs.view(-1).contiguous())
        del head
        self.final_norm = (1.0 + 0.02 * torch.randn(H, generator=gen, device=dev)).bfloat16()
        self.rope = rope_table(cfg.max_position, D, cfg.rope_theta, dev)
        return self

    def _shard_qkv(self, qw, sc):
        """Column shard of the fused [q | k | v] projection for this rank."""
        cfg, sh = self.cfg, self.shape
        D = cfg.head_dim
        q0 = self.rank * sh.hq_local * D
        cols = [torch.arange(q0, q0 + sh.hq_local * D, device=qw.device)]
        kv_heads = sh.kv_heads_of(self.rank, cfg.num_kv_heads)
        for base in (cfg.q_size, cfg.q_size + cfg.kv_size):
            for h in kv_heads:
                cols.append(torch.arange(base + h * D, base + (h + 1) * D, device=qw.device))
        idx = torch.cat(cols)
        return qw[:, idx].contiguous(), sc[:, idx].contiguous()

    def _shard_rows(self, qw, sc, k_local):
        """Row (K) shard for a row-parallel projection."""
        if self.tp == 1:
            return qw, sc
        k0 = self.rank * k_local
        return (qw[k0 // 8:(k0 + k_local) // 8].contiguous(),
                sc[k0 // 128:(k0 + k_local) // 128].contiguous())

    def _shard_gate_up(self, qw, sc):
        if self.tp == 1:
            return qw, sc
        I, il = self.cfg.intermediate, self.shape.inter_local
        r = self.rank
        idx = torch.cat([torch.arange(r * il, (r + 1) * il), torch.arange(I + r * il, I + (r + 1) * il)]).to(qw.device)
        return qw[:, idx].contiguous(), sc[:, idx].contiguous()

    # ------------------------------------------------------------- forward
    def _all_reduce(self, t: torch.Tensor) -> torch.Tensor:
        if self.tp > 1:
            self.comm.all_reduce(t)
        return t

    def embed(self, ids: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        x = ops.embed_int8(ids, self.embed_codes, self.embed_scales, start=self.vocab_start, out=out)
        return self._all_reduce(x)

    def _skip_attention(self, qkv: torch.Tensor, inp: StepInputs, cache: torch.Tensor,
                        lay: skip_layers.SkipLayout) -> torch.Tensor:
        """A skip layer's attention (``kv.skip_layers``): RoPE, the plain-dtype
        store and the paged attention in torch, on the same page ids and
        causal rule as the K8/V4 kernels. ``qkv`` is ``[T, hq + 2 hkv, D]``."""
        hq, hkv = self.shape.hq_local, self.shape.hkv_local
        q = skip_layers.apply_rope(qkv[:, :hq], self.rope, inp.positions)
        k = skip_layers.apply_rope(qkv[:, hq:hq + hkv], self.rope, inp.positions)
        skip_layers.store(cache, lay, inp.slots, k, qkv[:, hq + hkv:])
        return skip_layers.paged_attention(q, cache, lay, inp.block_table, inp.seq_lens, inp.cu_q, inp.positions,
                                           inp.max_q_len, self.shape.gqa_local, q_ends=inp.q_ends)

    def _cp_attention(self, q: torch.Tensor, inp: StepInputs, cache: torch.Tensor, layer: int) -> torch.Tensor:
        """Attention under context parallelism (see ``parallel.cp``)."""
        sh, cp = self.shape, self.cp
        hkv, gqa = sh.hkv_local, sh.gqa_local
        if not inp.is_decode:
            cp.sync(self.device)  # every rank's KV of this chunk is written
            return ops.prefill_attn_cp(q, inp.cu_q, inp.seq_lens, inp.block_table, cp.layer_caches(layer), hkv, gqa,
                                       inp.max_q_len, q_pos=inp.q_pos)
        B = inp.cu_q.numel() - 1
        nsplit = max(2, inp.nsplit)
        rank_floats = ops.decode_ws_floats(B, hkv, nsplit, inp.max_q_len, gqa)
        if cp.peer is not None and cp.peer.fits(rank_floats):
            # partials exchanged by the attention kernel itself (multicast stores)
            return cp.peer.attention(q, inp.cu_q, inp.cp_local_lens, inp.cp_local_bt, cache, hkv, gqa,
                                     inp.max_q_len, nsplit, q_ends=inp.q_ends)
        ws = torch.empty(rank_floats, dtype=torch.float32, device=self.device)
        ops.decode_attn(q, inp.cu_q, inp.cp_local_lens, inp.cp_local_bt, cache, hkv, gqa, inp.max_q_len,
                        nsplit=nsplit, ws=ws, q_ends=inp.q_ends)
        out = torch.empty_like(q)
        return ops.decode_combine_ranks(cp.all_gather(ws), rank_floats, inp.cu_q, cp.world, nsplit, hkv, gqa,
                                        inp.max_q_len, out)

    def _layer(self, L: LayerWeights, x: torch.Tensor, residual: torch.Tensor | None, inp: StepInputs,
               cache: torch.Tensor, ws, defer: bool, sync=None, tag: str = "layers", layer: int = -1):
        """One decoder layer. ``x`` may be fp32 sums left by the previous
        layer's GEMM (split-K partials, or this rank's copy of a fused
        all-reduce, then ``sync`` says when they are complete); they are
        finished inside the input norm. Returns (x, residual, sync)."""
        cfg, sh = self.cfg, self.shape
        T = inp.input_ids.shape[0]
        D = cfg.head_dim
        hq, hkv = sh.hq_local, sh.hkv_local
        splitk_ws = ws.splitk if ws is not None else None
        # the fused all-reduce epilogue belongs to the int4 GEMM (INT8 islands use NCCL)
        far = self.fused_ar if (self.fused_ar is not None and self.fused_ar.fits(T, cfg.hidden)
                                and isinstance(L.o, Int4Linear) and isinstance(L.down, Int4Linear)) else None
        # ---- attention block
        with stage(tag + ".input_norm"):
            if residual is None:
                residual = x.clone()
                h = ops.rmsnorm(x, L.input_norm, cfg.rms_eps)
            else:
                h = ops.rmsnorm(x, L.input_norm, cfg.rms_eps, residual=residual, sync=sync)
        skip = self.skip_kv.get(layer) if self.skip_kv else None
        with stage(tag + ".gemm_qkv"):
            # split-K at decode sizes: the fp32 sums go straight to rope_store,
            # which finishes them (bf16 rounding) and zeroes the accumulator
            qkv = L.qkv(h, ws=splitk_ws, defer=skip is None)
        if skip is None:
            q = torch.empty((T, hq, D), dtype=torch.bfloat16, device=self.device)
            with stage(tag + ".rope_store"):
                ops.rope_store(qkv, self.rope, inp.positions, q, inp.slots, cache, hq, hkv)
        with stage(tag + ".attn"):
            if skip is not None:
                a = self._skip_attention(qkv.reshape(T, hq + 2 * hkv, D), inp, cache, skip)
            elif self.cp is not None:
                a = self._cp_attention(q, inp, cache, layer)
            elif inp.is_decode:
                with attention_span("decode"):
                    a = ops.decode_attn(q, inp.cu_q, inp.seq_lens, inp.block_table, cache, hkv, sh.gqa_local,
                                        inp.max_q_len, nsplit=inp.nsplit, q_ends=inp.q_ends,
                                        ws=(ws.attn if ws is not None else None))
            else:
                with attention_span("prefill"):
                    a = ops.prefill_attn(q, inp.cu_q, inp.seq_lens, inp.block_table, cache, hkv, sh.gqa_local,
                                         inp.max_q_len)
        a = a.view(T, hq * D)
        with stage(tag + ".o_proj"):
            if far is not None:
                # TP: the all-reduce runs inside the GEMM epilogue (NVLS multicast adds)
                x, sync_o = far.gemm(L.o, 0, x=a)
            else:
                # single GPU: leave split-K partials for the fused norm below to finish
                x = L.o(a, ws=splitk_ws, defer=defer)
                sync_o = None
        if far is None:
            with stage(tag + ".all_reduce"):
                self._all_reduce(x)
        # ---- MLP block
        w4a8 = uses_w4a8(L.gate_up.name, T, self.w4a8) and L.gate_up.supports_w4a8 and L.down.supports_w4a8
        note_gemm_branch(L.gate_up.name, T, "w4a8" if w4a8 else "w4a16")
        if w4a8:
            with stage(tag + ".post_norm"):
                hq8, hs = ops.rmsnorm(x, L.post_norm, cfg.rms_eps, residual=residual, quant=True, sync=sync_o)
            with stage(tag + ".gate_up"):
                gu = L.gate_up(xq=hq8, xs=hs)
            with stage(tag + ".act"):
                aq, as_ = ops.silu_mul(gu, quant=True)
            with stage(tag + ".down"):
                if far is not None:
                    x, sync_d = far.gemm(L.down, 1, xq=aq, xs=as_)
                else:
                    x = L.down(xq=aq, xs=as_)
                    sync_d = None
        else:
            with stage(tag + ".post_norm"):
                h = ops.rmsnorm(x, L.post_norm, cfg.rms_eps, residual=residual, sync=sync_o)
            with stage(tag + ".gate_up"):
                # decode GEMV: the fp32 sums stay in the workspace for silu_mul
                gu = L.gate_up(h, ws=splitk_ws, defer=True)
            with stage(tag + ".act"):
                act = ops.silu_mul(gu)
            with stage(tag + ".down"):
                if far is not None:
                    x, sync_d = far.gemm(L.down, 1, x=act)
                else:
                    x = L.down(act, ws=splitk_ws, defer=defer)
                    sync_d = None
        if far is None:
            with stage(tag + ".all_reduce"):
                self._all_reduce(x)
        return x, residual, sync_d

    def _final_norm(self, x, residual, norm_w, rows: torch.Tensor | None, sync=None) -> torch.Tensor:
        cfg = self.cfg
        if x.dtype == torch.float32 or rows is None:
            # fp32 sums (or every row wanted): finish them in the norm over all rows
            h = ops.rmsnorm(x, norm_w, cfg.rms_eps, residual=residual, sync=sync)
            return h if rows is None else h.index_select(0, rows)
        xs = x.index_select(0, rows)
        rs = residual.index_select(0, rows)
        return ops.rmsnorm(xs, norm_w, cfg.rms_eps, residual=rs)

    def forward(self, inp: StepInputs, kv_caches: list[torch.Tensor], ws=None,
                all_rows: bool = False) -> torch.Tensor:
        """Run every layer; returns the final-normed hidden rows ``inp.logit_rows``
        (every row with ``all_rows``, as the MTP drafter needs)."""
        T = inp.input_ids.shape[0]
        if (self.sp is not None and not inp.is_decode and not all_rows and self.cp is None and not self.skip_kv
                and self.sp.fits(T, self.cfg.hidden) and self._sp_linears()):
            return self._forward_sp(inp, kv_caches)
        with stage("embed"):
            x = self.embed(inp.input_ids)
        residual = None
        sync = None
        defer = self.tp == 1
        for li, L in enumerate(self.layers):
            x, residual, sync = self._layer(L, x, residual, inp, kv_caches[li], ws, defer, sync, "layers.%d" % li,
                                            li)
        with stage("final_norm"):
            return self._final_norm(x, residual, self.final_norm, None if all_rows else inp.logit_rows, sync)

    def _sp_linears(self) -> bool:
        return all(isinstance(lin, Int4Linear) for L in self.layers for lin in (L.qkv, L.o, L.gate_up, L.down))

    def _forward_sp(self, inp: StepInputs, kv_caches: list[torch.Tensor]) -> torch.Tensor:
        """Tensor-parallel prefill with the residual stream sharded by token rows
        between the fused GEMM -> reduce-scatter and all-gather -> GEMM kernels
        (``parallel.seq_parallel``). Same math as ``_layer``; returns the
        final-normed rows ``inp.logit_rows`` on every rank."""
        cfg, sh, sp = self.cfg, self.shape, self.sp
        T = inp.input_ids.shape[0]
        D = cfg.head_dim
        hq, hkv = sh.hq_local, sh.hkv_local
        sp.begin(T)
        with stage("embed"):
            x = self.embed(inp.input_ids)  # vocab-parallel lookup, summed over the group
        for li, L in enumerate(self.layers):
            tag = "layers.%d" % li
            with stage(tag + ".input_norm"):
                if li == 0:
                    sp.norm_push(L.input_norm, cfg.rms_eps, gather=0, x_local=x[sp.row0:sp.row0 + sp.nrows])
                else:
                    sp.norm_push(L.input_norm, cfg.rms_eps, gather=0, slot=1)
            with stage(tag + ".gemm_qkv"):
                qkv = sp.gemm_ag(L.qkv, 0)
            q = torch.empty((T, hq, D), dtype=torch.bfloat16, device=self.device)
            with stage(tag + ".rope_store"):
                ops.rope_store(qkv, self.rope, inp.positions, q, inp.slots, kv_caches[li], hq, hkv)
            with stage(tag + ".attn"), attention_span("prefill"):
                a = ops.prefill_attn(q, inp.cu_q, inp.seq_lens, inp.block_table, kv_caches[li], hkv, sh.gqa_local,
                                     inp.max_q_len)
            with stage(tag + ".o_proj"):
                sp.gemm_rs(L.o, 0, x=a.view(T, hq * D))
            w4a8 = uses_w4a8(L.gate_up.name, T, self.w4a8) and L.gate_up.supports_w4a8 and L.down.supports_w4a8
            note_gemm_branch(L.gate_up.name, T, "w4a8" if w4a8 else "w4a16")
            gather = 1 if w4a8 else 2
            with stage(tag + ".post_norm"):
                sp.norm_push(L.post_norm, cfg.rms_eps, gather=gather, slot=0)
            with stage(tag + ".gate_up"):
                gu = sp.gemm_ag(L.gate_up, gather)
            with stage(tag + ".act"):
                if w4a8:
                    aq, as_ = ops.silu_mul(gu, quant=True)
                else:
                    act = ops.silu_mul(gu)
            with stage(tag + ".down"):
                if w4a8:
                    sp.gemm_rs(L.down, 1, xq=aq, xs=as_)
                else:
                    sp.gemm_rs(L.down, 1, x=act)
        with stage("final_norm"):
            local = sp.final_norm(self.final_norm, cfg.rms_eps, slot=1)
            return sp.gather_rows(local, inp.logit_rows, self.comm)

    # ---------------------------------------------------------------- MTP
    def init_mtp(self, seed: int = 1) -> "DenseModel":
        """Random-init the MTP draft module (one decoder layer of the same shape).

        Structure of the multi-token-prediction head served by the reference's
        ``--speculative-config mtp/6`` (``k8v4_v030/launch.sh:193``): the
        embedding of the next token and the target's final hidden state are
        normed separately, concatenated and projected back to ``hidden``
        (``eh_proj``, a column-parallel GPTQ linear), run through one decoder
        layer with its own KV cache, normed, and scored by the shared lm_head.
        """
        cfg, sh = self.cfg, self.shape
        dev = self.device
        gen = torch.Generator(device=dev).manual_seed(seed + 7919)
        H = cfg.hidden
        # eh_proj: [2H -> H]; under TP every rank holds all of it (it feeds the replicated residual)
        eh_q, eh_s = _rand_int4(2 * H, H, gen, dev)
        qkv_q, qkv_s = self._shard_qkv(*_rand_int4(H, cfg.q_size + 2 * cfg.kv_size, gen, dev))
        o_q, o_s = self._shard_rows(*_rand_int4(cfg.q_size, H, gen, dev), sh.hq_local * cfg.head_dim)
        gu_q, gu_s = self._shard_gate_up(*_rand_int4(H, 2 * cfg.intermediate, gen, dev))
        dn_q, dn_s = self._shard_rows(*_rand_int4(cfg.intermediate, H, gen, dev), sh.inter_local)
        pre = "mtp.layers.0."

        def nw():
            return (1.0 + 0.02 * torch.randn(H, generator=gen, device=dev)).bfloat16()

        self.mtp = MTPWeights(
            enorm=nw(), hnorm=nw(), norm=nw(),
            eh_proj=Int4Linear("mtp.eh_proj", eh_q, eh_s),
            layer=LayerWeights(
                input_norm=nw(), post_norm=nw(),
                qkv=Int4Linear(pre + "self_attn.qkv_proj", qkv_q, qkv_s),
                o=Int4Linear(pre + "self_attn.o_proj", o_q, o_s),
                gate_up=Int4Linear(pre + "mlp.gate_up_proj", gu_q, gu_s),
                down=Int4Linear(pre + "mlp.down_proj", dn_q, dn_s)),
        )
        return self

    def mtp_forward(self, hidden: torch.Tensor, ids: torch.Tensor, inp: StepInputs, cache: torch.Tensor,
                    ws=None) -> torch.Tensor:
        """One MTP pass over ``T`` rows: ``hidden`` [T, H] (the target's, or the
        previous draft's, final-normed state at position p) and ``ids`` [T] (the
        token at p + 1). Writes the MTP KV at ``inp.slots``; returns the MTP's
        final-normed hidden [T, H] (its next-token logits come from the lm_head)."""
        cfg, M = self.cfg, self.mtp
        T = ids.shape[0]
        H = cfg.hidden
        e = self.embed(ids)
        cat = torch.empty((T, 2 * H), dtype=torch.bfloat16, device=self.device)
        ops.rmsnorm(e, M.enorm, cfg.rms_eps, out=cat[:, :H])
        ops.rmsnorm(hidden, M.hnorm, cfg.rms_eps, out=cat[:, H:])
        splitk_ws = ws.splitk if ws is not None else None
        x = M.eh_proj(cat, ws=splitk_ws)
        x, residual, sync = self._layer(M.layer, x, None, inp, cache, ws, defer=self.tp == 1, tag="mtp",
                                        layer=len(self.layers))
        return self._final_norm(x, residual, M.norm, None, sync)

    def logits(self, hidden: torch.Tensor) -> torch.Tensor:
        """Local vocab shard logits ``[rows, V/tp]`` (bf16)."""
        with stage("lm_head"):
            q, s = ops.quant_rows(hidden)
            return self.lm_head(q, s)

    def greedy(self, hidden: torch.Tensor) -> torch.Tensor:
        """Greedy token ids ``[rows]`` (int64), reduced over vocab shards."""
        lg = self.logits(hidden)
        with stage("sampler.argmax"):
            val, idx = ops.argmax(lg, offset=self.vocab_start)
            if self.tp > 1:
                val, idx = self.comm.argmax_reduce(val, idx)
        return idx

    # ------------------------------------------------------------ reference
    def reference_forward(self, inp: StepInputs, kv_caches_cpu: list[torch.Tensor]):
        """fp32 torch reference of :meth:`forward` (TP1) for tests."""
        from ..kv.oracle import attention_ref
        from ..kv.pack import gather_sequence, store_tokens
        cfg = self.cfg
        H, D = cfg.hidden, cfg.head_dim
        ids = inp.input_ids.cpu()
        x = (self.embed_codes.cpu()[ids].bfloat16() * self.embed_scales.cpu()[ids].view(-1, 1).bfloat16())
        residual = None
        sh = self.shape
        cu = inp.cu_q.cpu().tolist()
        lens = inp.seq_lens.cpu().tolist()
        bt = inp.block_table.cpu()
        pos = inp.positions.cpu()
        rope = self.rope.cpu()

        def norm(v, w, res):
            if res is not None:
                v = (v.float() + res.float()).bfloat16()
            vf = v.float()
            y = (vf * torch.rsqrt(vf.pow(2).mean(-1, keepdim=True) + cfg.rms_eps)).bfloat16()
            return (w.cpu().float() * y.float()).bfloat16(), v

        def rot(t):
            c = rope[pos, : D // 2].unsqueeze(1)
            s = rope[pos, D // 2:].unsqueeze(1)
            a, b = t[..., : D // 2].float(), t[..., D // 2:].float()
            return torch.cat([a * c - b * s, b * c + a * s], -1).bfloat16()

        for li, L in enumerate(self.layers):
            h, residual = norm(x, L.input_norm, residual) if residual is not None else (norm(x, L.input_norm, None)[0], x)
            qkv = (h.float() @ L.qkv.dense_t()).bfloat16()
            T = qkv.shape[0]
            qkv = qkv.view(T, sh.hq_local + 2 * sh.hkv_local, D)
            q = rot(qkv[:, : sh.hq_local])
            k = rot(qkv[:, sh.hq_local: sh.hq_local + sh.hkv_local])
            v = qkv[:, sh.hq_local + sh.hkv_local:]
            store_tokens(kv_caches_cpu[li], inp.slots.cpu(), k, v, self.layout)
            outs = []
            for b in range(len(lens)):
                qs = q[cu[b]:cu[b + 1]]
                ql = qs.shape[0]
                npg = (lens[b] + 15) // 16
                kd, vd = gather_sequence(kv_caches_cpu[li], bt[b, :npg].tolist(), lens[b], self.layout)
                ends = [lens[b] - ql + t + 1 for t in range(ql)]
                outs.append(attention_ref(qs.float(), kd, vd, ends, sh.gqa_local))
            a = torch.cat(outs, 0).bfloat16().view(T, -1)
            x = (a.float() @ L.o.dense_t()).bfloat16()
            h, residual = norm(x, L.post_norm, residual)
            gu = (h.float() @ L.gate_up.dense_t()).bfloat16()
            I = gu.shape[1] // 2
            act = (torch.nn.functional.silu(gu[:, :I].float()) * gu[:, I:].float()).bfloat16()
            x = (act.float() @ L.down.dense_t()).bfloat16()
        rows = inp.logit_rows.cpu()
        y, _ = norm(x[rows], self.final_norm, residual[rows])
        return y
