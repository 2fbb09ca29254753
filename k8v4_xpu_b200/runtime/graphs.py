"""Full-decode-only CUDA graphs.

One graph per (batch size, query width) in the capture list: the whole
decode forward (embedding, every layer's GEMMs, RoPE + KV write, split-K
attention, collectives) plus the lm_head and greedy sampling. Graph inputs
live in the workspace's persistent buffers; a step copies that step's
metadata into them from pinned host memory and replays. Capture sizes follow
the reference's FULL_DECODE_ONLY profile (multiples of the decode width,
``k8v4_v030/launch.sh:65-70``); prefill never runs inside a graph (the
reference raised if it tried, ``k8v4_v030/backend.py:290-291``).
"""
from __future__ import annotations

import numpy as np
import torch

from .. import ops
from ..models.dense import StepInputs
from .sampling import needs_logits


def decode_inputs(ws, B: int, w: int, nsplit: int) -> StepInputs:
    """StepInputs over the workspace's graph-stable buffers: B sequences x w tokens."""
    T = B * w
    return StepInputs(
        input_ids=ws.input_ids[:T], positions=ws.positions[:T], slots=ws.slots[:T],
        cu_q=ws.cu_q[: B + 1], seq_lens=ws.seq_lens[:B], block_table=ws.block_table[:B],
        logit_rows=ws.logit_rows[:T], max_q_len=w, is_decode=True, nsplit=nsplit,
    )


def prepare_benign(eng, B: int, w: int) -> None:
    """Capture-time metadata: every sequence one page long, no KV writes."""
    ws = eng.ws
    T = B * w
    ws.cu_q[: B + 1].copy_(torch.arange(0, T + 1, w, dtype=torch.int32, device=eng.device))
    ws.seq_lens[:B].fill_(w)
    ws.block_table[:B].zero_()
    rows = eng.__dict__.get("_bt_rows")
    if rows:  # the zeroed rows no longer hold the tables stage_decode_inputs copied
        for i in range(B):
            rows.pop(i, None)
    ws.slots[:T].fill_(-1)  # capture must not write into live KV pages
    ws.positions[:T].zero_()
    ws.input_ids[:T].zero_()
    ws.logit_rows[:T].copy_(torch.arange(T, device=eng.device))
    ws.write_en[:B].zero_()
    ws.forced_a[:B].zero_()


def stage_decode_inputs(eng, sched, B: int, w: int, forced_a=None) -> None:
    """Copy one decode step's metadata into the graph buffers.

    Row i*w + j of the batch is token j of sequence i (its last token, then its
    drafts). Padding sequences (B > real batch) repeat a one-page context with
    every KV write dropped (slot -1, write_en 0); their block-table row keeps
    whatever valid page ids it held.

    Block-table rows are copied incrementally: the device row of batch slot i
    remembers (sequence, table version, pages copied), and a step sends only
    the pages appended since (a decode step usually sends none). A changed
    table (new sequence in the slot, replaced block, truncation) is rewritten.
    """
    ws = eng.ws
    T = B * w
    B_real = len(sched.chunks)
    ids = np.zeros(T, np.int64)
    pos = np.zeros(T, np.int64)
    slots = np.full(T, -1, np.int64)
    lens = np.full(B, w, np.int32)  # padding sequences: one page
    blocks = eng.blocks
    rows = eng.__dict__.setdefault("_bt_rows", {})
    updates = []  # (row, first page, pages)
    for i, c in enumerate(sched.chunks):
        seq = c.seq
        toks = [seq.last_token] + seq.draft
        ids[i * w:(i + 1) * w] = toks[:w]
        pos[i * w:(i + 1) * w] = np.arange(c.start, c.start + w)
        for j in range(w):
            slots[i * w + j] = blocks.slot(seq.seq_id, c.start + j)
        lens[i] = c.start + w
        ver = blocks.version.get(seq.seq_id, 0)
        n = blocks.num_pages(seq.seq_id)
        st = rows.get(i)
        start = st[2] if (st is not None and st[0] == seq.seq_id and st[1] == ver and st[2] <= n) else 0
        if n > start:
            updates.append((i, start, blocks.pages_from(seq.seq_id, start)))
        rows[i] = (seq.seq_id, ver, n)
    n64 = 3 * T + 2 * B
    pin64 = eng._pin_i64[:n64].numpy()
    pin64[:T], pin64[T:2 * T], pin64[2 * T:3 * T] = ids, pos, slots
    pin64[3 * T:3 * T + B] = [1 if i < B_real else 0 for i in range(B)]
    pin64[3 * T + B:] = 0 if forced_a is None else np.concatenate([forced_a, np.zeros(B - len(forced_a), np.int64)])
    n32 = (B + 1) + B
    pin32 = eng._pin_i32.numpy()
    pin32[: B + 1] = np.arange(0, T + 1, w)
    pin32[B + 1: 2 * B + 1] = lens
    off = n32
    table_bytes = 0
    for i, first, pages in updates:
        k = len(pages)
        pin32[off:off + k] = pages
        ws.block_table[i, first:first + k].copy_(eng._pin_i32[off:off + k], non_blocking=True)
        off += k
        table_bytes += 4 * k
    g64 = eng._pin_i64[:n64].to(eng.device, non_blocking=True)
    g32 = eng._pin_i32[:n32].to(eng.device, non_blocking=True)
    ws.input_ids[:T].copy_(g64[:T], non_blocking=True)
    ws.positions[:T].copy_(g64[T:2 * T], non_blocking=True)
    ws.slots[:T].copy_(g64[2 * T:3 * T], non_blocking=True)
    ws.write_en[:B].copy_(g64[3 * T:3 * T + B], non_blocking=True)
    ws.forced_a[:B].copy_(g64[3 * T + B:], non_blocking=True)
    ws.cu_q[: B + 1].copy_(g32[: B + 1], non_blocking=True)
    ws.seq_lens[:B].copy_(g32[B + 1: 2 * B + 1], non_blocking=True)
    eng.h2d_bytes += n64 * 8 + n32 * 4 + table_bytes


class DecodeGraphs:
    def __init__(self, engine, widths: tuple[int, ...] | None = None):
        self.engine = engine
        cfg = engine.cfg
        self.width = 1 + cfg.speculative_tokens
        sizes = cfg.capture_sizes or tuple(range(1, cfg.max_num_seqs + 1))
        self.sizes = sorted(set(int(s) for s in sizes if 1 <= s <= cfg.max_num_seqs))
        self.graphs: dict[tuple[int, int], tuple[torch.cuda.CUDAGraph, torch.Tensor, int]] = {}
        self.pool = None
        self.captured = False
        self.kernels: dict[tuple[int, int], int] = {}  # our kernel launches per replay

    def can_run(self, sched) -> bool:
        """Uniform decode batches that fit a captured size and take the
        argmax (a step with a request that samples or asks for
        log-probabilities runs eagerly)."""
        B = len(sched.chunks)
        widths = {c.num_tokens for c in sched.chunks}
        return (len(widths) == 1 and next(iter(widths)) in (1, self.width) and B <= max(self.sizes)
                and not any(needs_logits(c.seq.params) for c in sched.chunks))

    def capture(self, widths: tuple[int, ...] | None = None) -> None:
        eng = self.engine
        from .engine import decode_splits
        widths = widths or tuple(sorted({1, self.width}))
        ws = eng.ws
        stream = torch.cuda.Stream(device=eng.device)
        for w in widths:
            for B in self.sizes:
                nsplit = decode_splits(eng.max_pages, B, eng.layout.hkv)
                prepare_benign(eng, B, w)
                inp = decode_inputs(ws, B, w, nsplit)
                stream.wait_stream(torch.cuda.current_stream(eng.device))
                with torch.cuda.stream(stream):
                    for _ in range(2):  # warm-up (kernel attributes, allocator)
                        hid = eng.model.forward(inp, eng.kv_caches, ws)
                        out = eng.model.greedy(hid)
                torch.cuda.current_stream(eng.device).wait_stream(stream)
                g = torch.cuda.CUDAGraph()
                before = ops.LAUNCHES
                with torch.cuda.graph(g, pool=self.pool, stream=stream):
                    hid = eng.model.forward(inp, eng.kv_caches, ws)
                    out = eng.model.greedy(hid)
                self.kernels[(B, w)] = ops.LAUNCHES - before
                if self.pool is None:
                    self.pool = g.pool()
                self.graphs[(B, w)] = (g, out, nsplit)
        torch.cuda.synchronize(eng.device)
        self.captured = True

    def release(self) -> None:
        """Drop every graph (graphs holding NCCL calls must go before the process group)."""
        self.graphs.clear()
        self.pool = None
        self.captured = False

    def run(self, sched) -> np.ndarray:
        eng = self.engine
        if not self.captured:
            self.capture()
        B_real = len(sched.chunks)
        w = sched.chunks[0].num_tokens
        B = next(s for s in self.sizes if s >= B_real)
        g, out, _nsplit = self.graphs[(B, w)]
        stage_decode_inputs(eng, sched, B, w)
        g.replay()
        n = B_real * w
        host = eng._pin_out[:n]
        host.copy_(out[:n], non_blocking=True)
        torch.cuda.current_stream(eng.device).synchronize()
        eng.d2h_bytes += n * 8
        return host.numpy().copy()
