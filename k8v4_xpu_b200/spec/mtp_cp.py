"""MTP speculative decoding under context parallelism.

The reference serves ``--speculative-config mtp/6`` on every launcher profile
(``k8v4_v030/launch.sh:193-194``); its long-context profile shards nothing by
position, so this combination has no counterpart there. Here the KV pages of
every sequence, the MTP layer's included, are sharded by page across the CP
ranks (``parallel.cp``), and one speculative step runs on every rank as:

1. verify: the target forward over the ``B x (k + 1)`` rows ``[last, d1..dk]``
   with replicated GEMMs. Each row's KV goes to the owner of its page only.
   Each rank's decode attention covers its own pages; a row at position p
   sees the prefix of the rank's local keys that lie at or before p (the
   per-row visible ends ``q_ends``, :func:`parallel.cp.local_keys`). The
   partials of all ranks are then merged as in plain CP decode;
2. greedy rejection and the MTP catch-up over the same rows, as on one GPU
   (``spec.mtp``);
3. drafts 2..k, one row per sequence per step. Slots and local key counts
   are computed on the device from the accepted count, because the host does
   not know it until the step ends.

The result vector ``(targets, accepted, drafts)`` is broadcast from CP rank 0
before the host reads it, so every rank commits the same tokens.

After a prefill step each rank runs the MTP layer over the prompt rows it
owns (their MTP KV stays local). For a prompt that completed, the owner of
its last row contributes that row's MTP hidden state to a sum over the CP
group (the other ranks add zeros), and every rank drafts from it.

Steps run eagerly (no CUDA graphs), like the rest of CP decode.
"""
from __future__ import annotations

import numpy as np
import torch

from ..models.dense import StepInputs
from ..parallel.cp import PAGE, local_keys, local_slots
from ..runtime.block_manager import CapacityError
from .mtp import MTPSpeculator, next_token_rows


class CPMTPSpeculator(MTPSpeculator):
    def __init__(self, engine, k: int, forced_accept_mean: float | None = None, seed: int = 0):
        super().__init__(engine, k, forced_accept_mean, seed)
        if self.topk_log is not None:
            raise ValueError("MTP top-k logging runs without context parallelism")
        self.use_graphs = False

    # ------------------------------------------------------------ host side
    def _block_rows(self, seqs) -> tuple[torch.Tensor, torch.Tensor, int]:
        """Block ids of each sequence [B, W] (zero padded) and their count [B]
        on the device. Under CP a rank's local page list of a sequence is its
        block list: block b holds logical page b * C + rank on this rank."""
        eng = self.eng
        tables = [eng.blocks.tables[s.seq_id] for s in seqs]
        W = max(1, max(len(t) for t in tables))
        a = np.zeros((len(tables), W), np.int32)
        for i, t in enumerate(tables):
            a[i, :len(t)] = t
        n = np.array([len(t) for t in tables], np.int64)
        eng.h2d_bytes += a.nbytes + n.nbytes
        return torch.from_numpy(a).to(eng.device), torch.from_numpy(n).to(eng.device), W

    def _splits(self, W: int, B: int) -> int:
        from ..runtime.engine import decode_splits
        return max(2, decode_splits(W, B, self.eng.layout.hkv))

    def verify_inputs(self, sched) -> tuple[StepInputs, torch.Tensor, torch.Tensor]:
        """StepInputs of the verify rows on this rank, with the block rows the
        drafts' slots are computed from."""
        eng, cp = self.eng, self.eng.cp
        w = self.w
        chunks = sched.chunks
        B = len(chunks)
        T = B * w
        C, r = cp.world, cp.rank
        ids = np.zeros(T, np.int64)
        pos = np.zeros(T, np.int64)
        slots = np.full(T, -1, np.int64)
        q_ends = np.zeros(T, np.int32)
        lens = np.zeros(B, np.int32)
        local_lens = np.zeros(B, np.int32)
        enc = []
        for i, c in enumerate(chunks):
            seq = c.seq
            blocks = eng.blocks.tables[seq.seq_id]
            ids[i * w:(i + 1) * w] = ([seq.last_token] + list(seq.draft))[:w]
            for j in range(w):
                p = c.start + j
                pos[i * w + j] = p
                if p // (PAGE * C) < len(blocks):
                    slots[i * w + j] = cp.slot(blocks, p)
                q_ends[i * w + j] = local_keys(p + 1, r, C)
            lens[i] = c.start + w
            local_lens[i] = local_keys(c.start + w, r, C)
            enc.append(cp.encoded_pages(blocks, c.start + w))
        blk, nblk, W = self._block_rows([c.seq for c in chunks])
        We = max(1, max(len(e) for e in enc))
        table = np.zeros((B, We), np.int32)
        for i, e in enumerate(enc):
            table[i, :len(e)] = e
        dev = eng.device
        gqa = eng.model.shape.gqa_local
        inp = StepInputs(
            input_ids=torch.from_numpy(ids).to(dev), positions=torch.from_numpy(pos).to(dev),
            slots=torch.from_numpy(slots).to(dev),
            cu_q=torch.arange(0, T + 1, w, dtype=torch.int32, device=dev),
            seq_lens=torch.from_numpy(lens).to(dev), block_table=torch.from_numpy(table).to(dev),
            logit_rows=torch.arange(T, dtype=torch.int64, device=dev), max_q_len=w,
            is_decode=w * gqa <= 64, q_ends=torch.from_numpy(q_ends).to(dev),
            q_pos=torch.from_numpy(pos.astype(np.int32)).to(dev), cp_local_bt=blk,
            cp_local_lens=torch.from_numpy(local_lens).to(dev), nsplit=self._splits(W, B))
        eng.h2d_bytes += ids.nbytes + pos.nbytes * 2 + slots.nbytes + q_ends.nbytes + lens.nbytes * 2 + table.nbytes
        return inp, blk, nblk

    def step(self, sched) -> list:
        """One speculative decode step for every sequence in ``sched``."""
        eng = self.eng
        chunks = sched.chunks
        B = len(chunks)
        for c in chunks:
            if len(c.seq.draft) != self.k:
                c.seq.draft = (c.seq.draft + [c.seq.tokens[-1]] * self.k)[: self.k]
        inp, blk, nblk = self.verify_inputs(sched)
        forced = None
        if self.forced:
            forced = torch.from_numpy(self.forced_counts(B)).to(eng.device)
        out = self._verify(inp, blk, nblk, B, forced, [c.seq for c in chunks])
        eng.cp.broadcast_(out)
        res = out.cpu().numpy()
        eng.d2h_bytes += res.size * 8
        w, k = self.w, self.k
        return self.commit(sched, res[:B * w].reshape(B, w), res[B * w:B * w + B], res[B * w + B:].reshape(B, k))

    # ----------------------------------------------------------- device body
    def _verify(self, inp: StepInputs, blk, nblk, B: int, forced, seqs=None) -> torch.Tensor:
        """Returns int64 ``[B*w (targets) | B (accepted) | B*k (next drafts)]``."""
        eng, m, ws = self.eng, self.eng.model, self.eng.ws
        w = self.w
        T = B * w
        hid = m.forward(inp, eng.kv_caches, ws, all_rows=True)
        ids = inp.input_ids.view(B, w)
        d = ids[:, 1:]
        t, a = self._accept(hid, ids, B, seqs, forced)
        j = torch.arange(w, device=eng.device).view(1, w)
        nxt = torch.cat([d, t[:, -1:]], 1)
        catch_ids = torch.where(j < a.view(B, 1), nxt, t).reshape(T)
        mh = m.mtp_forward(hid, catch_ids, inp, eng.kv_caches[-1], ws)
        rows = torch.arange(B, device=eng.device) * w + a
        h = mh.index_select(0, rows)
        d1 = self._propose(h)
        base = inp.positions.index_select(0, rows)
        drafts = self.draft_loop(h, d1, base, blk, nblk, inp.nsplit)
        return torch.cat([t.reshape(T), a, drafts.reshape(B * self.k)])

    def draft_loop(self, h: torch.Tensor, d1: torch.Tensor, base: torch.Tensor, blk: torch.Tensor,
                   nblk: torch.Tensor, nsplit: int) -> torch.Tensor:
        """Drafts 2..k under CP: row i at position ``base[i] + step``; its MTP
        KV goes to the page's owner, and each rank's attention sees its own
        keys up to that position. Returns drafts [B, k]."""
        eng, m, cp = self.eng, self.eng.model, self.eng.cp
        B = d1.shape[0]
        cu = torch.arange(B + 1, dtype=torch.int32, device=eng.device)
        rows = torch.arange(B, dtype=torch.int64, device=eng.device)
        drafts = [d1]
        d = d1
        for step in range(1, self.k):
            pos = base + step
            inp = StepInputs(input_ids=d, positions=pos, slots=local_slots(blk, nblk, pos, cp.rank, cp.world),
                             cu_q=cu, seq_lens=(pos + 1).to(torch.int32), block_table=blk, logit_rows=rows,
                             max_q_len=1, is_decode=True, nsplit=nsplit, cp_local_bt=blk,
                             cp_local_lens=local_keys(pos + 1, cp.rank, cp.world).to(torch.int32))
            h = m.mtp_forward(h, d, inp, eng.kv_caches[-1], eng.ws)
            d = self._propose(h)
            drafts.append(d)
        return torch.stack(drafts, 1)

    # ---------------------------------------------------------- after prefill
    def after_prefill_cp(self, sched, inp: StepInputs, hid_all: torch.Tensor, all_tok: np.ndarray) -> None:
        """MTP catch-up over this rank's rows of a prefill step, then drafts
        for the prompts that completed. ``all_tok`` [len(chunks)] holds the
        token sampled for each chunk (summed over ranks; 0 where none)."""
        eng, m, cp = self.eng, self.eng.model, self.eng.cp
        T = hid_all.shape[0]
        ids = np.zeros(T, np.int64)
        finals = []  # (chunk, row on the owner, owner)
        r = 0
        for ci, c in enumerate(sched.chunks):
            seq = c.seq
            end = c.start + c.num_tokens
            owned = [p for p in range(c.start, end) if cp.owner(p) == cp.rank]
            tok = int(all_tok[ci]) if c.needs_logits else None
            if c.is_prefill and owned:
                nxt = next_token_rows(seq.tokens, c.start, end, seq.prefill_target, tok)
                ids[r:r + len(owned)] = [nxt[p - c.start] for p in owned]
            if c.is_prefill and c.needs_logits:
                finals.append((c, r + len(owned) - 1, cp.owner(end - 1)))
            r += len(owned)
        dev_ids = torch.from_numpy(ids).to(eng.device)
        eng.h2d_bytes += ids.nbytes
        mh = m.mtp_forward(hid_all, dev_ids, inp, eng.kv_caches[-1], eng.ws)
        live = []
        for c, row, owner in finals:
            try:
                eng.blocks.ensure(c.seq.seq_id, c.start + c.num_tokens + self.k)
                live.append((c, row, owner))
            except CapacityError:
                c.seq.draft = [c.seq.tokens[-1]] * self.k  # no room to draft: verify rejects these
        if not live:
            return
        B = len(live)
        h = torch.zeros((B, mh.shape[1]), dtype=mh.dtype, device=eng.device)
        mine = [(i, row) for i, (_, row, owner) in enumerate(live) if owner == cp.rank]
        if mine:
            at = torch.tensor([i for i, _ in mine], dtype=torch.int64, device=eng.device)
            h.index_copy_(0, at, mh.index_select(0, torch.tensor([row for _, row in mine], dtype=torch.int64,
                                                                   device=eng.device)))
        cp.sum_(h)  # the owner's row; the other ranks add zeros
        d1 = self._propose(h)
        base = torch.tensor([c.start + c.num_tokens - 1 for c, _, _ in live], dtype=torch.int64, device=eng.device)
        blk, nblk, W = self._block_rows([c.seq for c, _, _ in live])
        drafts = self.draft_loop(h, d1, base, blk, nblk, self._splits(W, B))
        cp.broadcast_(drafts)
        host = drafts.cpu().numpy()
        eng.d2h_bytes += host.size * 8
        for i, (c, _, _) in enumerate(live):
            c.seq.draft = [int(x) for x in host[i]]
