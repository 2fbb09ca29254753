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
all-gather, or with ``K8V4_CP_COMBINE=peer`` multicast stores from the decode
attention kernel (``parallel.cp_combine``). Tensor parallelism inside each
CP rank (CP x TP, ``parallel.groups``) shards the model over the TP group as
in the plain engine; the CP exchange then runs between the ranks that hold
the same KV heads. MTP under CP is not supported yet.
"""
from __future__ import annotations

import numpy as np
import torch

from ..models.dense import StepInputs
from ..parallel.cp import PAGE, CPGroup
from ..parallel.cp_combine import PeerCombine, cp_combine_mode, max_slot_floats
from .block_manager import BlockManager, CapacityError
from .engine import LLMEngine, decode_splits


class CPEngine(LLMEngine):
    """``cp``: this rank's CP group. With TP inside each CP rank
    (``tensor_parallel_size`` > 1), ``comm`` is the TP group's communicator
    and ``rank`` this process's TP rank (``parallel.groups``)."""

    def __init__(self, cfg, model_cfg, cp: CPGroup, rank: int = 0, comm=None):
        if cfg.speculative_tokens:
            raise NotImplementedError("context parallelism runs without MTP")
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
        if cp_combine_mode() == "peer" and cp.world > 1:
            sh = self.model.shape
            try:
                cp.peer = PeerCombine(cp.group, self.device,
                                      max_slot_floats(cfg.max_num_seqs, sh.hkv_local, 1, sh.gqa_local))
            except Exception as e:  # no multicast on this box: NCCL all-gather
                import logging
                logging.getLogger("k8v4").warning("peer partial exchange unavailable (%s); using NCCL", e)

    def _alloc_cache(self) -> None:
        cfg = self.cfg
        page_bytes = self.layout.page_bytes
        n_layers = len(self.model.layers)
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

    def _plain_step(self, sched):
        inp, owned = self._build_inputs(sched)
        n_logit = sum(1 for c in sched.chunks if c.needs_logits)
        hidden = self.model.forward(inp, self.kv_caches, self.ws)
        if sched.is_decode_only:
            tokens = self._sample(hidden) if n_logit else np.zeros(0, np.int64)
        else:
            # the owner of each prompt's last token samples it; the others add zeros
            vec = torch.zeros(len(sched.chunks), dtype=torch.int64, device=self.device)
            if owned:
                ids = self.model.greedy(hidden)
                vec[torch.tensor([ci for ci, _ in owned], device=self.device)] = ids
            self.cp.sum_(vec)
            all_tok = vec.cpu().numpy()
            self.d2h_bytes += all_tok.size * 8
            tokens = np.array([all_tok[i] for i, c in enumerate(sched.chunks) if c.needs_logits], np.int64)
        return self._commit(sched, tokens)
