"""K8/V4 attention backend with the shape of a vLLM V1 backend.

The reference registers ``Xe2K8V4AttentionBackend`` with vLLM
(``k8v4_v030/backend.py:448-486``): a metadata builder that classifies each
batch, and an implementation whose KV update (``do_kv_cache_update``) runs
separately from ``forward``. Decode batches (uniform packed q_len) run as one
launch over all requests; prefill runs per batch; prefill inside a CUDA
graph capture raises (``backend.py:290-291``), since only decode steps are
captured (FULL_DECODE_ONLY).

This module keeps that contract over the b200 kernels:

* cache: one ``uint8 [num_pages, hkv * 3232]`` tensor per layer
  (``get_kv_cache_shape``), 202 bytes per token per KV head;
* ``K8V4MetadataBuilder.build`` -> :class:`K8V4Metadata` (device tensors +
  the decode / prefill decision and the split-K factor);
* ``K8V4AttentionImpl.do_kv_cache_update`` -> ``k8v4.kv_store``;
  ``forward`` -> ``k8v4.decode_attn`` or ``k8v4.prefill_attn``.

It is the integration surface for an external engine (the vLLM plugin in
``k8v4_xpu_b200.registry`` points vLLM at it); the built-in engine calls the
same ops directly from the model.
"""
from __future__ import annotations

import dataclasses
import math

import torch

from .. import ops
from ..kv.layout import CACHE_DTYPE
from .plan import decode_workspace_floats, require_decoder, uniform_packed_q_len

NUM_SMS = 148


@dataclasses.dataclass
class K8V4Metadata:
    cu_q: torch.Tensor          # [B+1] int32
    seq_lens: torch.Tensor      # [B] int32 (context incl. this step's tokens)
    block_table: torch.Tensor   # [B, W] int32 kernel pages
    slot_mapping: torch.Tensor  # [T] int64
    max_q_len: int
    num_decode_tokens: int
    is_decode: bool
    nsplit: int = 1
    q_ends: torch.Tensor | None = None  # [T] int32 per-token visible ends (MTP trees)


class K8V4AttentionBackend:
    accept_output_buffer = True

    @staticmethod
    def get_name() -> str:
        return "K8V4_B200"

    @staticmethod
    def get_supported_kv_cache_dtypes() -> list[str]:
        return [CACHE_DTYPE]

    @staticmethod
    def get_kv_cache_shape(num_blocks: int, block_size: int, num_kv_heads: int, head_size: int,
                           cache_dtype_str: str = CACHE_DTYPE) -> tuple[int, int]:
        if cache_dtype_str != CACHE_DTYPE:
            raise ValueError("K8V4 backend serves kv_cache_dtype=%s" % CACHE_DTYPE)
        if head_size != 128 or block_size % 16:
            raise ValueError("K8V4 b200 pages: head_size 128, block_size a multiple of 16")
        return (num_blocks * (block_size // 16), num_kv_heads * 3232)

    @staticmethod
    def state_bytes_per_token(num_kv_heads: int) -> int:
        """202 bytes per KV head per token (the reference's 396 at D = 256)."""
        return 202 * num_kv_heads

    @staticmethod
    def get_metadata_builder_cls():
        return K8V4MetadataBuilder

    @staticmethod
    def get_impl_cls():
        return K8V4AttentionImpl


class K8V4MetadataBuilder:
    def __init__(self, num_heads: int, num_kv_heads: int, device="cuda", max_splits: int = 64):
        self.layout = require_decoder(128, num_heads, num_kv_heads)
        self.device = torch.device(device)
        self.max_splits = max_splits

    def splits_for(self, max_pages: int, nseq: int) -> int:
        tiles = max(1, (max_pages + 7) // 8)
        return int(max(1, min(NUM_SMS // max(1, nseq * self.layout.hkv), tiles, self.max_splits)))

    def build(self, query_lens: list[int], seq_lens: list[int], block_tables: list[list[int]],
              slot_mapping: list[int], q_ends: list[int] | None = None) -> K8V4Metadata:
        if not (len(query_lens) == len(seq_lens) == len(block_tables)):
            raise ValueError("one query length, context length and block table per request")
        for q, n in zip(query_lens, seq_lens):
            if q < 1 or q > n:
                raise ValueError("each request needs 1 <= q_len <= seq_len")
        B = len(query_lens)
        cu = [0]
        for q in query_lens:
            cu.append(cu[-1] + int(q))
        if len(slot_mapping) != cu[-1]:
            raise ValueError("slot_mapping needs one slot per query token")
        W = max(1, max(len(t) for t in block_tables))
        bt = torch.zeros((B, W), dtype=torch.int32)
        for i, t in enumerate(block_tables):
            if (int(seq_lens[i]) + 15) // 16 > len(t):
                raise ValueError("request %d: block table covers fewer pages than seq_len" % i)
            bt[i, :len(t)] = torch.tensor(t, dtype=torch.int32)
        q = uniform_packed_q_len(query_lens, self.layout.gqa)
        dev = self.device
        md = K8V4Metadata(
            cu_q=torch.tensor(cu, dtype=torch.int32, device=dev),
            seq_lens=torch.tensor(seq_lens, dtype=torch.int32, device=dev),
            block_table=bt.to(dev), slot_mapping=torch.tensor(slot_mapping, dtype=torch.int64, device=dev),
            max_q_len=max(query_lens), num_decode_tokens=cu[-1] if q is not None else 0, is_decode=q is not None,
            q_ends=torch.tensor(q_ends, dtype=torch.int32, device=dev) if q_ends is not None else None)
        if md.is_decode:
            md.nsplit = self.splits_for(W, B)
        return md


class K8V4AttentionImpl:
    def __init__(self, num_heads: int, head_size: int, scale: float | None, num_kv_heads: int,
                 alibi_slopes=None, sliding_window=None, kv_cache_dtype: str = CACHE_DTYPE,
                 logits_soft_cap=None, attn_type: str = "decoder", sinks=None):
        if kv_cache_dtype != CACHE_DTYPE:
            raise ValueError("K8V4 backend serves kv_cache_dtype=%s" % CACHE_DTYPE)
        self.layout = require_decoder(head_size, num_heads, num_kv_heads, sliding_window, alibi_slopes,
                                      logits_soft_cap, attn_type, sinks)
        self.num_heads, self.num_kv_heads, self.head_size = num_heads, num_kv_heads, head_size
        self.scale = float(scale) if scale is not None else 1.0 / math.sqrt(head_size)
        self._ws = None

    def _workspace(self, md: K8V4Metadata, device) -> torch.Tensor | None:
        if md.nsplit <= 1:
            return None
        need = decode_workspace_floats(md.seq_lens.numel(), self.num_kv_heads, md.nsplit, md.max_q_len,
                                       self.layout.gqa)
        if self._ws is None or self._ws.numel() < need or self._ws.device != device:
            if torch.cuda.is_current_stream_capturing():
                raise RuntimeError("decode workspace must be sized before CUDA graph capture")
            self._ws = torch.empty(need, dtype=torch.float32, device=device)
        return self._ws

    def do_kv_cache_update(self, key: torch.Tensor, value: torch.Tensor, kv_cache: torch.Tensor,
                           slot_mapping: torch.Tensor) -> None:
        """Quantize and write this step's K/V rows ([T, hkv, 128] bf16) into the pages."""
        ops.kv_store(key, value, slot_mapping, kv_cache, self.num_kv_heads)

    def forward(self, query: torch.Tensor, key: torch.Tensor | None, value: torch.Tensor | None,
                kv_cache: torch.Tensor, md: K8V4Metadata, output: torch.Tensor | None = None) -> torch.Tensor:
        """``query`` [T, hq, 128] bf16 (rotated). With key/value given, writes
        them first. Returns / fills ``output`` [T, hq, 128] bf16."""
        if key is not None and value is not None:
            self.do_kv_cache_update(key, value, kv_cache, md.slot_mapping)
        hkv, gqa = self.num_kv_heads, self.layout.gqa
        if md.is_decode:
            out = ops.decode_attn(query, md.cu_q, md.seq_lens, md.block_table, kv_cache, hkv, gqa, md.max_q_len,
                                  nsplit=md.nsplit, q_ends=md.q_ends, ws=self._workspace(md, query.device),
                                  sm_scale=self.scale)
        else:
            if torch.cuda.is_available() and torch.cuda.is_current_stream_capturing():
                raise RuntimeError("K8V4 prefill cannot run inside a CUDA graph (FULL_DECODE_ONLY capture)")
            out = ops.prefill_attn(query, md.cu_q, md.seq_lens, md.block_table, kv_cache, hkv, gqa, md.max_q_len,
                                   sm_scale=self.scale)
        if output is not None:
            output.copy_(out)
            return output
        return out
