"""MTP speculative decoding: one draft layer, k drafts, (k + 1)-token verify.

The reference serves ``--speculative-config mtp/6`` (``k8v4_v030/launch.sh
:193``) through stock vLLM: the target verifies ``[last, d1..d6]`` as a
7-row query per sequence inside the FULL_DECODE_ONLY graph, a greedy
rejection sampler keeps the longest draft prefix that matches the target's
argmax, and the MTP layer proposes the next 6 drafts one token at a time
(its attention runs the same K8/V4 backend with ``q_len = 1``).

Here one decode step is ONE CUDA graph per batch size:

1. target forward over the ``B x 7`` verify rows, greedy ids ``t[B, 7]``;
2. on-device rejection: ``a = number of leading j with d[j+1] == t[j]``
   (or, in the forced benchmark mode, ``a`` read from an input buffer that
   the host fills from a seeded Bernoulli chain);
3. MTP catch-up over the same 7 rows: row j pairs the target hidden at
   position ``start + j`` with the token at ``start + j + 1`` (``d[j+1]`` for
   j < a, ``t[a]`` at j = a), writing the MTP layer's own KV; rows past ``a``
   write slots the next step overwrites;
4. draft 1 = argmax of the MTP output at row ``a``; drafts 2..k each run the
   MTP layer on one row per sequence, with positions and KV slots computed on
   the device from ``a`` and the block table.

A step with a request that samples (temperature > 0) or asks for
log-probabilities runs the same body eagerly: such sequences are verified by
speculative sampling against the target's sampling distribution, and their
entry ``t[a]`` holds the token drawn there (``_accept``).

The host reads back ``(t, a, drafts)`` in one copy, emits ``d[1..a] + t[a]``
and rolls the sequence's valid length back to ``start + a + 1``: KV written
past it is dead and overwritten by later steps (rollback by length, as the
reference's backend does with ``seq_lens``).
"""
from __future__ import annotations

import dataclasses

import numpy as np
import torch

from ..models.dense import StepInputs
from ..runtime.block_manager import CapacityError
from ..runtime import sampling
from ..runtime.sampling import generator_for, samples, speculative_sample
from ..runtime.engine import stream_sync
from ..runtime.graphs import decode_inputs, prepare_benign, stage_decode_inputs


def next_token_rows(tokens, start: int, end: int, prefill_len: int, sampled: int | None) -> list[int]:
    """The MTP input of prefill rows ``start .. end-1``: the token at p + 1
    for row p, and for the last row of the whole prefill (``end ==
    prefill_len``) the token sampled there. The prefilled tokens are the
    prompt, or after a recompute preemption prompt + output."""
    nxt = list(tokens[start + 1:min(end + 1, prefill_len)])
    if end >= prefill_len:
        nxt.append(sampled)
    return nxt


def forced_accept_prob(mean_len: float, k: int) -> float:
    """Per-position acceptance probability p of a Bernoulli chain (stop at the
    first rejection, at most k accepted) whose mean accepted LENGTH
    ``E[1 + accepted] = sum_{i=0..k} p^i`` equals ``mean_len``."""
    if not 1.0 <= mean_len <= k + 1:
        raise ValueError("mean accepted length must lie in [1, %d]" % (k + 1))
    if mean_len == k + 1:
        return 1.0
    lo, hi = 0.0, 1.0
    for _ in range(100):
        mid = 0.5 * (lo + hi)
        if sum(mid ** i for i in range(k + 1)) < mean_len:
            lo = mid
        else:
            hi = mid
    return 0.5 * (lo + hi)


@dataclasses.dataclass
class SpecStats:
    """Acceptance accounting, exported as the ``vllm:spec_decode_*`` counters."""

    k: int
    num_drafts: int = 0           # verify steps x sequences
    num_draft_tokens: int = 0
    num_accepted_tokens: int = 0
    accepted_per_pos: list[int] = dataclasses.field(default_factory=list)

    def __post_init__(self):
        if not self.accepted_per_pos:
            self.accepted_per_pos = [0] * self.k

    def record(self, accepted: int) -> None:
        self.num_drafts += 1
        self.num_draft_tokens += self.k
        self.num_accepted_tokens += accepted
        for i in range(accepted):
            self.accepted_per_pos[i] += 1

    @property
    def mean_accepted_length(self) -> float:
        return 1.0 + self.num_accepted_tokens / max(1, self.num_drafts)


class MTPSpeculator:
    _GOLDEN = 0.6180339887498949  # fractional part of the golden ratio
    def __init__(self, engine, k: int, forced_accept_mean: float | None = None, seed: int = 0):
        if k < 1:
            raise ValueError("MTP needs at least one draft token")
        self.eng = engine
        self.k = k
        self.w = k + 1
        self.forced = forced_accept_mean is not None
        self.p = forced_accept_prob(forced_accept_mean, k) if self.forced else None
        self.rng = np.random.default_rng(seed)
        self._u0 = float(self.rng.random())  # forced mode: start of the golden-ratio sequence
        self._n = 0
        self.stats = SpecStats(k)
        self.use_graphs = engine.cfg.cuda_graphs
        cfg = engine.cfg
        sizes = cfg.capture_sizes or tuple(range(1, cfg.max_num_seqs + 1))
        # capture sizes are given in rows (7, 14, ...) or in sequences
        self.sizes = sorted({(s // self.w if s % self.w == 0 and s >= self.w else s) for s in sizes
                             if 1 <= s <= max(cfg.max_num_seqs, cfg.max_num_seqs * self.w)} & set(
            range(1, cfg.max_num_seqs + 1))) or list(range(1, cfg.max_num_seqs + 1))
        self.graphs: dict[int, tuple[torch.cuda.CUDAGraph, torch.Tensor]] = {}
        self.pool = None
        self.kernels: dict[int, int] = {}
        from .topk_log import TopKLogger
        self.topk_log = TopKLogger.from_env()  # draft top-k logging (eager drafting, TP1)
        if self.topk_log is not None:
            if engine.tp > 1:
                raise ValueError("MTP top-k logging runs at tensor parallel size 1")
            self.use_graphs = False
        self._topk: list = []  # (ids [B, 8], vals [B, 8]) per draft position of the current call
        self.lookahead = self.w  # KV slots past the verify window that drafting writes

    # ------------------------------------------------------------ forced mode
    def forced_counts(self, n: int) -> np.ndarray:
        """Accepted-draft counts of ``n`` sequences for one step.

        The count has the Bernoulli chain's distribution (``P(count >= i) =
        p^i``), drawn by inverting that tail at a quasi-random uniform ``u``
        (the additive golden-ratio sequence from a seeded start): ``count =
        #{i <= k : u < p^i}``. The sequence fills [0, 1) evenly, so the
        realized mean over a benchmark's few hundred rows sits on the
        configured mean instead of drifting by the sampling noise of
        independent draws."""
        u = (self._u0 + self._GOLDEN * (self._n + np.arange(n))) % 1.0
        self._n += n
        tails = self.p ** np.arange(1, self.k + 1)
        return (u[:, None] < tails[None, :]).sum(axis=1).astype(np.int64)

    # ------------------------------------------------------------ device body
    def _propose(self, h: torch.Tensor) -> torch.Tensor:
        """Next draft ids from MTP hidden rows (greedy; with top-k logging the
        drafter's top-8 of each position is kept too)."""
        m = self.eng.model
        if self.topk_log is None:
            return m.greedy(h)
        vals, ids = torch.topk(m.logits(h).float(), 8, dim=-1)
        ids = ids + m.vocab_start
        self._topk.append((ids, vals))
        return ids[:, 0].contiguous()

    def _draft_loop(self, h: torch.Tensor, d1: torch.Tensor, base: torch.Tensor, bt: torch.Tensor,
                    write_en: torch.Tensor, nsplit: int) -> torch.Tensor:
        """Drafts 2..k: one MTP row per sequence per step. ``base`` [B] is the
        position of the hidden row that produced ``d1``. Returns drafts [B, k]."""
        eng, m = self.eng, self.eng.model
        B = d1.shape[0]
        page = eng.layout.page
        cu = torch.arange(B + 1, dtype=torch.int32, device=eng.device)
        rows = torch.arange(B, dtype=torch.int64, device=eng.device)
        drafts = [d1]
        d = d1
        for step in range(1, self.k):
            pos = base + step
            pg = bt.gather(1, (pos // page).view(B, 1).to(torch.int64)).view(B).to(torch.int64)
            slot = torch.where(write_en > 0, pg * page + pos % page, torch.full_like(pos, -1))
            inp = StepInputs(input_ids=d, positions=pos, slots=slot, cu_q=cu, seq_lens=(pos + 1).to(torch.int32),
                             block_table=bt, logit_rows=rows, max_q_len=1, is_decode=True, nsplit=nsplit)
            h = m.mtp_forward(h, d, inp, eng.kv_caches[-1], eng.ws)
            d = self._propose(h)
            drafts.append(d)
        return torch.stack(drafts, 1)

    def _accept(self, hid: torch.Tensor, ids: torch.Tensor, B: int, seqs=None, forced=None):
        """Targets ``t`` [B, w] and accepted drafts ``a`` [B] of the verify rows.

        Greedy sequences keep the longest draft prefix that equals the
        target's argmax (``t`` holds the argmax). Sampling sequences (an eager
        step) run speculative sampling against the target's sampling
        distribution (``runtime.sampling.speculative_sample``), and ``t[i, a]``
        holds the token drawn there, so the commit emits ``d[:a] + t[a]`` for
        both kinds. ``forced`` [B]: the benchmark's accepted counts."""
        m = self.eng.model
        w = self.w
        d = ids[:, 1:]
        if forced is not None or not seqs or not any(sampling.needs_logits(s.params) for s in seqs):
            t = m.greedy(hid).view(B, w)
            a = forced if forced is not None else (d == t[:, :-1]).to(torch.int64).cumprod(1).sum(1)
            return t, a
        lg = m.logits(hid)
        if self.eng.tp > 1:
            lg = m.comm.all_gather(lg, dim=1)
        lg = lg.reshape(B, w, -1)  # the lm_head may return a view over padded vocab rows
        pick = lg
        if any(sampling.has_processors(s.params) for s in seqs):
            # row j follows the committed output and drafts 1..j
            pick = lg.float().clone()
            for i, s in enumerate(seqs):
                if sampling.has_processors(s.params):
                    dj = d[i].tolist()
                    for j in range(w):
                        pick[i, j] = sampling.process_row(lg[i, j], s.prompt, list(s.output) + dj[:j],
                                                              s.params, holder=s)
        t = torch.argmax(pick.float(), dim=-1)
        a = (d == t[:, :-1]).to(torch.int64).cumprod(1).sum(1)
        stash = sampling.stash_of(self.eng)
        for i, s in enumerate(seqs):
            if samples(s.params):
                g = generator_for(s, self.eng.cfg.seed, self.eng.device)
                ai, x = speculative_sample(pick[i], d[i], s.params, g)
                a[i] = ai
                t[i, ai] = x
            if sampling.wants_logprobs(s.params):  # one entry per token the commit will emit
                ai = int(a[i])
                toks = d[i, :ai].tolist() + [int(t[i, ai])]
                stash[s.seq_id] = [sampling.logprob_entry(lg[i, j], tok, s.params.logprobs)
                                   for j, tok in enumerate(toks)]
        return t, a

    def _body(self, B: int, nsplit: int, seqs=None) -> torch.Tensor:
        """The whole speculative decode step on the graph buffers (``seqs``:
        the real sequences of an eager step, for the ones that sample).

        Returns int64 ``[B*w (targets) | B (accepted) | B*k (next drafts)]``."""
        eng, m, ws = self.eng, self.eng.model, self.eng.ws
        w, k = self.w, self.k
        T = B * w
        inp = decode_inputs(ws, B, w, nsplit)
        hid = m.forward(inp, eng.kv_caches, ws, all_rows=True)     # [T, H]
        ids = inp.input_ids.view(B, w)
        d = ids[:, 1:]
        t, a = self._accept(hid, ids, B, seqs, ws.forced_a[:B] if self.forced else None)
        j = torch.arange(w, device=eng.device).view(1, w)
        nxt = torch.cat([d, t[:, -1:]], 1)
        catch_ids = torch.where(j < a.view(B, 1), nxt, t).reshape(T)
        mh = m.mtp_forward(hid, catch_ids, inp, eng.kv_caches[-1], ws)
        rows = torch.arange(B, device=eng.device) * w + a
        h = mh.index_select(0, rows)
        d1 = self._propose(h)
        base = inp.positions.index_select(0, rows)
        drafts = self._draft_loop(h, d1, base, inp.block_table, ws.write_en[:B], nsplit)
        return torch.cat([t.reshape(T), a, drafts.reshape(B * k)])

    def capture(self) -> None:
        from .. import ops
        eng = self.eng
        from ..runtime.engine import decode_splits
        stream = torch.cuda.Stream(device=eng.device)
        for B in self.sizes:
            nsplit = decode_splits(eng.max_pages, B, eng.layout.hkv)
            prepare_benign(eng, B, self.w)
            stream.wait_stream(torch.cuda.current_stream(eng.device))
            with torch.cuda.stream(stream):
                for _ in range(2):
                    self._body(B, nsplit)
            torch.cuda.current_stream(eng.device).wait_stream(stream)
            g = torch.cuda.CUDAGraph()
            before = ops.LAUNCHES
            with torch.cuda.graph(g, pool=self.pool, stream=stream):
                out = self._body(B, nsplit)
            self.kernels[B] = ops.LAUNCHES - before
            if self.pool is None:
                self.pool = g.pool()
            self.graphs[B] = (g, out)
        torch.cuda.synchronize(eng.device)

    def release(self) -> None:
        self.graphs.clear()
        self.pool = None

    # ------------------------------------------------------------- host side
    def step(self, sched) -> list:
        """One decode step for every sequence in ``sched`` (all width k + 1)."""
        eng = self.eng
        from ..runtime.engine import decode_splits
        chunks = sched.chunks
        B_real = len(chunks)
        B = next((s for s in self.sizes if s >= B_real), None)
        if B is None:
            raise RuntimeError("MTP batch %d exceeds the largest capture size" % B_real)
        for c in chunks:
            if len(c.seq.draft) != self.k:
                c.seq.draft = (c.seq.draft + [c.seq.tokens[-1]] * self.k)[: self.k]
        if self.use_graphs and not self.graphs:
            self.capture()  # before staging: capture fills the buffers with benign metadata
        forced = self.forced_counts(B_real) if self.forced else None
        stage_decode_inputs(eng, sched, B, self.w, forced)
        self._topk = []
        if self.use_graphs and not any(sampling.needs_logits(c.seq.params) for c in chunks):
            g, out = self.graphs[B]
            g.replay()
        else:  # eager: no graphs, or a request that samples or asks for log-probabilities
            out = self._body(B, decode_splits(eng.max_pages, B, eng.layout.hkv), [c.seq for c in chunks])
        n = out.numel()
        host = eng._pin_out[:n]
        host.copy_(out, non_blocking=True)
        stream_sync(eng.device)
        eng.d2h_bytes += n * 8
        res = host.numpy().copy()
        w, k = self.w, self.k
        t = res[: B * w].reshape(B, w)
        acc = res[B * w: B * w + B]
        nd = res[B * w + B:].reshape(B, k)
        if self.topk_log is not None:
            for i, c in enumerate(sched.chunks):
                prev = getattr(c.seq, "draft_topk", None)
                if prev is not None:
                    self.topk_log.record(c.seq.seq_id, c.seq.draft, prev[0], prev[1], t[i].tolist(), int(acc[i]))
            self.topk_log.end_step()
            self._stash_topk([c.seq for c in sched.chunks])
        return self.commit(sched, t, acc, nd)

    def _stash_topk(self, seqs) -> None:
        """Keep each sequence's draft top-k for the next verify step's log line."""
        if not self._topk:
            return
        ids = torch.stack([a for a, _ in self._topk], 1).cpu()   # [B, k, 8]
        vals = torch.stack([b for _, b in self._topk], 1).cpu()
        for i, seq in enumerate(seqs):
            seq.draft_topk = (ids[i].tolist(), vals[i].tolist())
        self._topk = []

    def commit(self, sched, t: np.ndarray, acc: np.ndarray, drafts: np.ndarray) -> list:
        eng = self.eng
        finished = []
        for i, c in enumerate(sched.chunks):
            seq = c.seq
            a = int(acc[i])
            self.stats.record(a)
            emitted = list(seq.draft[:a]) + [int(t[i, a])]
            # valid KV now covers [last, d1..da]; slots past it are dead (rollback by length)
            seq.computed = c.start + a + 1
            seq.draft = [int(x) for x in drafts[i]]
            stopped = False
            for tok in emitted:
                seq.output.append(tok)
                sampling.record(eng, seq)
                eng.stats["generated_tokens"] += 1
                if eng._should_stop(seq, tok):
                    reason = "length" if len(seq.output) >= seq.params.max_tokens else "stop"
                    eng.scheduler.finish(seq, reason)
                    finished.append(seq)
                    stopped = True
                    break
            sampling.stash_of(eng).pop(seq.seq_id, None)  # entries past a stop are dropped
            if not stopped:
                eng.blocks.publish(seq.seq_id, seq.tokens, seq.computed)
        return finished

    # ----------------------------------------------------------- after prefill
    def after_prefill(self, sched, inp: StepInputs, hid_all: torch.Tensor, tokens: np.ndarray) -> None:
        """MTP catch-up over a prefill step's rows, then drafts for the
        sequences whose prompt just completed.

        Row r at position p pairs the target hidden state with the token at
        p + 1: the next prompt token, or the token sampled this step for the
        last prompt row.
        """
        eng, m = self.eng, self.eng.model
        T = hid_all.shape[0]
        ids = np.zeros(T, np.int64)
        finals = []  # (chunk, row, sampled token)
        r = 0
        k_tok = 0
        for c in sched.chunks:
            seq = c.seq
            n = c.num_tokens
            end = c.start + n
            if c.needs_logits:
                tok = int(tokens[k_tok])
                k_tok += 1
            else:
                tok = None
            if c.is_prefill:
                ids[r:r + n] = next_token_rows(seq.tokens, c.start, end, seq.prefill_target, tok)
                if c.needs_logits:
                    finals.append((c, r + n - 1))
            r += n
        pin = eng._pin_i64[:T].numpy()
        pin[:] = ids
        dev_ids = eng._pin_i64[:T].to(eng.device, non_blocking=True)
        eng.h2d_bytes += T * 8
        mh = m.mtp_forward(hid_all, dev_ids, inp, eng.kv_caches[-1], eng.ws)
        if not finals:
            stream_sync(eng.device)
            return
        live = []
        for c, row in finals:
            try:
                eng.blocks.ensure(c.seq.seq_id, c.start + c.num_tokens + self.k)
                live.append((c, row))
            except CapacityError:
                c.seq.draft = [c.seq.tokens[-1]] * self.k  # no room to draft: verify rejects these
        if not live:
            return
        B = len(live)
        rows = torch.tensor([row for _, row in live], dtype=torch.int64, device=eng.device)
        h = mh.index_select(0, rows)
        self._topk = []
        d1 = self._propose(h)
        base = torch.tensor([c.start + c.num_tokens - 1 for c, _ in live], dtype=torch.int64, device=eng.device)
        tables = [eng.blocks.page_table(c.seq.seq_id) for c, _ in live]
        W = max(len(tb) for tb in tables)
        bt = torch.zeros((B, W), dtype=torch.int32)
        for i, tb in enumerate(tables):
            bt[i, :len(tb)] = torch.tensor(tb, dtype=torch.int32)
        bt = bt.to(eng.device)
        from ..runtime.engine import decode_splits
        drafts = self._draft_loop(h, d1, base, bt, torch.ones(B, dtype=torch.int64, device=eng.device),
                                  decode_splits(eng.max_pages, B, eng.layout.hkv))
        host = drafts.cpu().numpy()
        eng.d2h_bytes += host.size * 8
        for i, (c, _) in enumerate(live):
            c.seq.draft = [int(x) for x in host[i]]
        if self.topk_log is not None:
            self._stash_topk([c.seq for c, _ in live])
