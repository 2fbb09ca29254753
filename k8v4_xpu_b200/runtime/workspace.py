"""Persistent device buffers reused by every forward (graph-stable addresses).

The reference kept its decode scratch in process-wide buffers allocated
before graph capture and only narrowed them per call (``k8v4_v030/
scratch.py:17-115``). Here the workspace holds the split-K fp32 accumulator
(kept all-zero between GEMMs: each split-K GEMM's finishing kernel clears
what it used), the decode attention partials, and the per-step input
buffers the CUDA graphs read.
"""
from __future__ import annotations

import torch

from .. import ops


class Workspace:
    def __init__(self, device, max_tokens: int, max_seqs: int, max_pages_per_seq: int, max_n: int,
                 heads: int, gqa: int, max_q_len: int, max_splits: int):
        self.device = torch.device(device)
        self.max_tokens = int(max_tokens)
        self.max_seqs = int(max_seqs)
        self.max_pages = int(max_pages_per_seq)
        # split-K accumulator for skinny GEMMs (rows <= 64)
        self.splitk = torch.zeros((min(64, max_tokens) * max_n,), dtype=torch.float32, device=self.device)
        self.attn = None
        if ops.available():
            n = ops.decode_ws_floats(max_seqs, heads, max_splits, max_q_len, gqa)
            self.attn = torch.empty(n, dtype=torch.float32, device=self.device)
        # graph input buffers
        self.input_ids = torch.zeros(max_tokens, dtype=torch.int64, device=self.device)
        self.positions = torch.zeros(max_tokens, dtype=torch.int64, device=self.device)
        self.slots = torch.zeros(max_tokens, dtype=torch.int64, device=self.device)
        self.cu_q = torch.zeros(max_seqs + 1, dtype=torch.int32, device=self.device)
        self.seq_lens = torch.zeros(max_seqs, dtype=torch.int32, device=self.device)
        self.block_table = torch.zeros((max_seqs, self.max_pages), dtype=torch.int32, device=self.device)
        self.logit_rows = torch.zeros(max_tokens, dtype=torch.int64, device=self.device)
        self.q_ends = torch.zeros(max_tokens, dtype=torch.int32, device=self.device)
        # MTP step inputs: per-sequence KV-write enable (0 for padding rows) and
        # the forced accepted-draft count of the benchmark acceptance mode
        self.write_en = torch.zeros(max_seqs, dtype=torch.int64, device=self.device)
        self.forced_a = torch.zeros(max_seqs, dtype=torch.int64, device=self.device)

