"""The serving engine under context parallelism (one process per GPU).

Every CP rank runs this engine on the same request stream (rank 0 serves
HTTP; followers mirror its commands, as under TP), so all ranks schedule the
same steps. What differs per rank (see ``parallel.cp``):

* the KV pool holds one page per CP block (page ``rank`` of every block), and
  every rank's pool is mapped into every process;
* a prefill step feeds each rank only the chunk tokens on its own pages; a
  rank with none runs one dummy row (no KV write, no logits) so that every
  rank takes the same collectives; the first token is sampled by the owner of
  the prompt's last token and summed across ranks;
* a decode step feeds every rank the new tokens (replicated GEMMs), the owner
  writes each token's KV, and attention merges every rank's partials.

Decode runs eagerly here. The per-layer partial exchange is an NCCL
all-gather (``K8V4_CP_COMBINE=nccl``) or, by default, multicast stores from the decode
attention kernel (``parallel.cp_combine``). Tensor parallelism inside each
CP rank (CP x TP, ``parallel.groups``) shards the model over the TP group as
in the plain engine; the CP exchange then runs between the ranks that hold
the same KV heads. MTP speculative decoding runs through
``spec.mtp_cp.CPMTPSpeculator`` (the MTP layer's pages are sharded like the
others).
"""
from __future__ import annotations

import os

import numpy as np
import torch

from ..models.dense import StepInputs
from ..parallel.cp import PAGE, CPGroup
from ..parallel.cp_combine import PeerCombine, cp_combine_mode, max_slot_floats
from .block_manager import CapacityError
from .engine import LLMEngine, decode_splits
from .sampling import needs_logits


class CPEngine(LLMEngine):
    """``cp``: this rank's CP group. With TP inside each CP rank
    (``tensor_parallel_size`` > 1), ``comm`` is the TP group's communicator
    and ``rank`` this process's TP rank (``parallel.groups``)."""

    def __init__(self, cfg, model_cfg, cp: CPGroup, rank: int = 0, comm=None):
        if cfg.tensor_parallel_size > 1 and comm is None:
            raise ValueError("tensor parallelism inside a CP group needs the TP group's communicator")
        if cfg.context_parallel_size != cp.world:
            raise ValueError("context_parallel_size %d != CP group size %d" % (cfg.context_parallel_size, cp.world))
        self.cp = cp
        cfg.cuda_graphs = False
        if cfg.block_size != PAGE * cp.world:
            cfg.block_size = PAGE * cp.world  # one CP block = one page on every rank
        super().__init__(cfg, model_cfg, comm=comm, rank=rank)
        self.model.cp = cp
        self.cp_rank = cp.rank
        if cfg.speculative_tokens:
            from ..spec.mtp_cp import CPMTPSpeculator
            self.mtp = CPMTPSpeculator(self, cfg.speculative_tokens, cfg.forced_accept_mean, cfg.seed)
        self.cp_graphs = CPDecodeGraphs(self) if cp_graphs_enabled() else None
        # shutdown paths release `graphs` before the process group goes
        self.graphs = self.cp_graphs
        if cp_combine_mode() == "peer" and cp.world > 1:
            sh = self.model.shape
            try:
                cp.peer = PeerCombine(cp.group, self.device,
                                      max_slot_floats(cfg.max_num_seqs, sh.hkv_local, 1 + cfg.speculative_tokens,
                                                      sh.gqa_local))
            except Exception as e:  # no multicast on this box: NCCL all-gather
                import logging
                logging.getLogger("k8v4").warning("peer partial exchange unavailable (%s); using NCCL", e)

    def _alloc_cache(self) -> None:
        cfg = self.cfg
        page_bytes = self.layout.page_bytes
        n_layers = len(self.model.layers) + (1 if self.model.mtp is not None else 0)
        if cfg.num_kv_blocks is not None:
            blocks = int(cfg.num_kv_blocks)
        else:
            free, total = torch.cuda.mem_get_info(self.device)
            budget = free - (1 - cfg.gpu_memory_utilization) * total - (4 << 30)
            blocks = int(budget // (page_bytes * n_layers))
            need = ((cfg.max_model_len + cfg.block_size - 1) // cfg.block_size + 1) * cfg.max_num_seqs
            blocks = max(1, min(blocks, need))
        if blocks * cfg.block_size < cfg.max_model_len:
            raise CapacityError("max_model_len %d exceeds the CP KV capacity of %d tokens"
                                % (cfg.max_model_len, blocks * cfg.block_size),
                                fit_tokens=blocks * cfg.block_size - 2)
        self.num_blocks = blocks
        self.kv_pool = self.cp.alloc_pool((n_layers, blocks, page_bytes), self.device)
        self.kv_caches = [self.kv_pool[i] for i in range(n_layers)]
        self.kv_capacity_tokens = blocks * cfg.block_size

    # ------------------------------------------------------------- inputs
    def _build_inputs(self, sched):
        cp, dev = self.cp, self.device
        chunks = sched.chunks
        decode = sched.is_decode_only
        ids, pos, slots, cu, lens, rows = [], [], [], [0], [], []
        bts, local_bts, local_lens = [], [], []
        owned_logit = []  # (chunk index, local row) of the logits this rank produces
        for ci, c in enumerate(chunks):
            seq = c.seq
            toks = seq.tokens
            blocks = self.blocks.tables[seq.seq_id]
            end = c.start + c.num_tokens
            feed = range(c.start, end)
            if not decode:
                feed = [p for p in feed if cp.owner(p) == cp.rank]
            for p in feed:
                ids.append(toks[p] if c.is_prefill else toks[-1])
                pos.append(p)
                slots.append(cp.slot(blocks, p))
            cu.append(len(ids))
            lens.append(end)
            bts.append(cp.encoded_pages(blocks, end))
            lp, lk = cp.local_pages(blocks, end)
            local_bts.append(lp or [0])
            local_lens.append(lk)
            if c.needs_logits and (decode or cp.owner(end - 1) == cp.rank):
                owned_logit.append((ci, len(ids) - 1))
        if not ids:  # this rank owns none of the chunk's tokens: one row that writes and samples nothing
            ids, pos, slots, cu = [0], [0], [-1], [0] + [1] * len(chunks)
        T = len(ids)
        B = len(chunks)

        def table(rows_):
            W = max(1, max(len(t) for t in rows_))
            a = np.zeros((B, W), np.int32)
            for i, t in enumerate(rows_):
                a[i, :len(t)] = t
            return torch.from_numpy(a).to(dev)

        max_q = max(int(cu[i + 1] - cu[i]) for i in range(B))
        inp = StepInputs(
            input_ids=torch.tensor(ids, dtype=torch.int64, device=dev),
            positions=torch.tensor(pos, dtype=torch.int64, device=dev),
            slots=torch.tensor(slots, dtype=torch.int64, device=dev),
            cu_q=torch.tensor(cu, dtype=torch.int32, device=dev),
            seq_lens=torch.tensor(lens, dtype=torch.int32, device=dev), block_table=table(bts),
            logit_rows=torch.tensor([r for _, r in owned_logit], dtype=torch.int64, device=dev),
            max_q_len=max(1, max_q), is_decode=decode,
            q_pos=torch.tensor(pos, dtype=torch.int32, device=dev),
            cp_local_bt=table(local_bts), cp_local_lens=torch.tensor(local_lens, dtype=torch.int32, device=dev))
        if decode:
            inp.nsplit = max(2, decode_splits(max(len(t) for t in local_bts), B, self.layout.hkv))
        self.h2d_bytes += T * 8 * 3 + B * 4 * 3
        return inp, owned_logit

    def _agree(self, ids: torch.Tensor) -> torch.Tensor:
        """Decode rows are replicated on every CP rank, but the fp32 atomics
        of a GEMM can sum in a different order on each, so a near-tie of two
        logits can break differently; CP rank 0's ids win."""
        return self.cp.broadcast_(ids)

    def _plain_step(self, sched):
        if self.cp_graphs is not None and sched.is_decode_only and self.cp_graphs.can_run(sched):
            return self._commit(sched, self.cp_graphs.run(sched))
        inp, owned = self._build_inputs(sched)
        n_logit = sum(1 for c in sched.chunks if c.needs_logits)
        hid_all = None
        if self.mtp is not None and not sched.is_decode_only:
            # the MTP layer catches up on every row this rank owns
            hid_all = self.model.forward(inp, self.kv_caches, self.ws, all_rows=True)
            hidden = hid_all.index_select(0, inp.logit_rows)
        else:
            hidden = self.model.forward(inp, self.kv_caches, self.ws)
        if sched.is_decode_only:
            seqs = [c.seq for c in sched.chunks if c.needs_logits]
            tokens = self._sample(hidden, seqs) if n_logit else np.zeros(0, np.int64)
        else:
            # the owner of each prompt's last token samples it; the others add zeros
            vec = torch.zeros(len(sched.chunks), dtype=torch.int64, device=self.device)
            if owned:
                ids = self._choose(hidden, [sched.chunks[ci].seq for ci, _ in owned])
                vec[torch.tensor([ci for ci, _ in owned], device=self.device)] = ids
            self.cp.sum_(vec)
            all_tok = vec.cpu().numpy()
            self.d2h_bytes += all_tok.size * 8
            tokens = np.array([all_tok[i] for i, c in enumerate(sched.chunks) if c.needs_logits], np.int64)
            if hid_all is not None:
                self.mtp.after_prefill_cp(sched, inp, hid_all, all_tok)
        return self._commit(sched, tokens)


def cp_graphs_enabled() -> bool:
    """``K8V4_CP_GRAPHS=1``: decode steps under CP replay captured CUDA graphs
    (off by default until the multi-GPU tests have run them)."""
    return os.environ.get("K8V4_CP_GRAPHS", "0") not in ("", "0")


class CPDecodeGraphs:
    """CUDA graphs of the CP decode step, one per batch size.

    Per step the host stages into graph-stable buffers the new tokens, their
    positions, this rank's KV slot of each (-1 where another rank owns the
    page), and this rank's page list and key count of each sequence. The
    split count is fixed per batch size (one wave of CTAs at the longest
    local page list), and the partial exchange (NCCL all-gather or the
    attention kernel's multicast stores) is captured with the rest of the
    step; every rank captures and replays the same graphs in the same order.
    Padding sequences hold no keys on any rank and write no KV.
    """

    def __init__(self, eng: "CPEngine"):
        self.eng = eng
        cfg = eng.cfg
        dev = eng.device
        self.sizes = list(range(1, cfg.max_num_seqs + 1))
        self.local_w = (eng.max_pages + eng.cp.world - 1) // eng.cp.world + 1
        B = cfg.max_num_seqs
        self.ids = torch.zeros(B, dtype=torch.int64, device=dev)
        self.pos = torch.zeros(B, dtype=torch.int64, device=dev)
        self.slots = torch.full((B,), -1, dtype=torch.int64, device=dev)
        self.cu = torch.arange(B + 1, dtype=torch.int32, device=dev)
        self.lens = torch.ones(B, dtype=torch.int32, device=dev)
        self.table = torch.zeros((B, 1), dtype=torch.int32, device=dev)
        self.rows = torch.arange(B, dtype=torch.int64, device=dev)
        self.local_bt = torch.zeros((B, self.local_w), dtype=torch.int32, device=dev)
        self.local_lens = torch.zeros(B, dtype=torch.int32, device=dev)
        self._pin64 = torch.zeros(3 * B, dtype=torch.int64, pin_memory=True)
        self._pin32 = torch.zeros(2 * B + B * self.local_w, dtype=torch.int32, pin_memory=True)
        self.graphs: dict[int, tuple] = {}
        self.pool = None

    def can_run(self, sched) -> bool:
        # the multicast exchange alternates two buffers per call; a captured
        # step keeps that alternation across replays only with an even count
        if self.eng.cp.peer is not None and len(self.eng.model.layers) % 2:
            return False
        return (len(sched.chunks) <= len(self.sizes) and all(c.num_tokens == 1 for c in sched.chunks)
                and not any(needs_logits(c.seq.params) for c in sched.chunks))

    def _inputs(self, B: int, nsplit: int) -> StepInputs:
        return StepInputs(
            input_ids=self.ids[:B], positions=self.pos[:B], slots=self.slots[:B], cu_q=self.cu[:B + 1],
            seq_lens=self.lens[:B], block_table=self.table[:B], logit_rows=self.rows[:B], max_q_len=1,
            is_decode=True, cp_local_bt=self.local_bt[:B], cp_local_lens=self.local_lens[:B], nsplit=nsplit)

    def _benign(self, B: int) -> None:
        self.slots[:B].fill_(-1)
        self.pos[:B].zero_()
        self.ids[:B].zero_()
        self.lens[:B].fill_(1)
        self.local_lens[:B].zero_()
        self.local_bt[:B].zero_()

    def capture(self, B: int) -> None:
        eng = self.eng
        nsplit = max(2, decode_splits(self.local_w, B, eng.layout.hkv))
        self._benign(B)
        inp = self._inputs(B, nsplit)
        stream = torch.cuda.Stream(device=eng.device)
        stream.wait_stream(torch.cuda.current_stream(eng.device))
        with torch.cuda.stream(stream):
            for _ in range(2):  # warm-up: kernel attributes, allocator, communicator
                out = eng._agree(eng.model.greedy(eng.model.forward(inp, eng.kv_caches, eng.ws)))
        torch.cuda.current_stream(eng.device).wait_stream(stream)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, pool=self.pool, stream=stream):
            out = eng._agree(eng.model.greedy(eng.model.forward(inp, eng.kv_caches, eng.ws)))
        if self.pool is None:
            self.pool = g.pool()
        torch.cuda.synchronize(eng.device)
        self.graphs[B] = (g, out)

    def run(self, sched) -> np.ndarray:
        eng, cp = self.eng, self.eng.cp
        B_real = len(sched.chunks)
        B = next(s for s in self.sizes if s >= B_real)
        if B not in self.graphs:
            self.capture(B)
        W = self.local_w
        p64 = self._pin64.numpy()
        p32 = self._pin32.numpy()
        p64[:3 * B] = 0
        p64[2 * B:3 * B] = -1
        p32[:2 * B + B * W] = 0
        p32[:B] = 1  # padding sequences: one key, none of it on this rank
        for i, c in enumerate(sched.chunks):
            seq = c.seq
            blocks = eng.blocks.tables[seq.seq_id]
            end = c.start + 1
            p64[i] = seq.tokens[-1]
            p64[B + i] = c.start
            p64[2 * B + i] = cp.slot(blocks, c.start)
            p32[i] = end
            pages, keys = cp.local_pages(blocks, end)
            if len(pages) > W:
                raise RuntimeError("sequence holds %d local pages, the graphs %d" % (len(pages), W))
            p32[B + i] = keys
            p32[2 * B + i * W: 2 * B + i * W + len(pages)] = pages
        g64 = self._pin64[:3 * B].to(eng.device, non_blocking=True)
        g32 = self._pin32[:2 * B + B * W].to(eng.device, non_blocking=True)
        self.ids[:B].copy_(g64[:B], non_blocking=True)
        self.pos[:B].copy_(g64[B:2 * B], non_blocking=True)
        self.slots[:B].copy_(g64[2 * B:3 * B], non_blocking=True)
        self.lens[:B].copy_(g32[:B], non_blocking=True)
        self.local_lens[:B].copy_(g32[B:2 * B], non_blocking=True)
        self.local_bt[:B].copy_(g32[2 * B:].view(B, W), non_blocking=True)
        eng.h2d_bytes += 3 * B * 8 + (2 * B + B * W) * 4
        g, out = self.graphs[B]
        g.replay()
        tokens = eng._pin_out[:B]
        tokens.copy_(out, non_blocking=True)
        torch.cuda.current_stream(eng.device).synchronize()
        eng.d2h_bytes += B_real * 8
        return tokens.numpy()[:B_real].copy()

    def release(self) -> None:
        """Drop every graph (they hold NCCL calls: before the process group goes)."""
        self.graphs.clear()
        self.pool = None
