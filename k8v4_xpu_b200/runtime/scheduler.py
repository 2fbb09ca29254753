"""Continuous-batching scheduler with chunked prefill.

Each step spends a token budget (``max_num_batched_tokens``, default 4,224 as
in the reference deployment, ``k8v4_v030/launch.sh:185``) decode-first:
every running sequence that is generating gets its decode tokens (1, or
1 + draft tokens under MTP), then the remaining budget goes to prefill chunks
of sequences that still have prompt tokens, in arrival order, admitting
waiting requests while ``max_num_seqs`` and the KV pool allow. A prompt
longer than the remaining budget is split into chunks across steps.
"""
from __future__ import annotations

import collections
import dataclasses
import enum
import itertools
import time

from .block_manager import BlockManager, CapacityError


class SeqStatus(enum.Enum):
    WAITING = "waiting"
    RUNNING = "running"
    FINISHED = "finished"


@dataclasses.dataclass
class SamplingParams:
    max_tokens: int = 16
    ignore_eos: bool = False
    stop_token_ids: tuple[int, ...] = ()
    temperature: float = 0.0  # 0: greedy decoding (the benchmark path); > 0: sampling
    top_p: float = 1.0        # nucleus sampling (1: off)
    top_k: int = 0            # top-k sampling (0: off)
    seed: int | None = None   # per-request generator seed (None: derived from the engine seed)
    logprobs: int | None = None  # None: off; N: each token's log-probability and the top N
    prompt_logprobs: int | None = None  # the same for the prompt tokens (no prefix-cache hits then)
    repetition_penalty: float = 1.0   # vLLM's penalties (1 / 0: off)
    presence_penalty: float = 0.0
    frequency_penalty: float = 0.0
    min_p: float = 0.0          # drop tokens below min_p x the top probability (0: off)
    logit_bias: dict | None = None  # token id -> bias added to its logit
    min_tokens: int = 0         # stop tokens are held back until the output is this long
    allowed_sequences: tuple | None = None  # guided choice: the output must be one of these token lists


@dataclasses.dataclass
class Sequence:
    seq_id: int
    prompt: list[int]
    params: SamplingParams
    output: list[int] = dataclasses.field(default_factory=list)
    status: SeqStatus = SeqStatus.WAITING
    computed: int = 0          # tokens whose KV is written
    cached_tokens: int = 0     # prompt tokens served by the prefix cache
    arrival: float = dataclasses.field(default_factory=time.monotonic)
    first_token_time: float | None = None
    finish_time: float | None = None
    finish_reason: str | None = None
    draft: list[int] = dataclasses.field(default_factory=list)  # MTP proposals for the next step
    prefill_start: float | None = None
    # tokens to prefill: the prompt, or after a recompute preemption every
    # token the sequence held (prompt + output so far)
    prefill_len: int | None = None
    generator: object = None   # torch.Generator of a sampling request (runtime.sampling)
    logprobs: list = dataclasses.field(default_factory=list)  # per output token, when requested
    prompt_logprobs: list = dataclasses.field(default_factory=list)  # per prompt token (None for the first)

    @property
    def tokens(self) -> "TokenView":
        """prompt + output without copying either (a 128K-token prompt made the
        concatenation a per-step cost): len(), indexing, slices (lists)."""
        return TokenView(self.prompt, self.output)

    @property
    def last_token(self) -> int:
        return self.output[-1] if self.output else self.prompt[-1]

    @property
    def num_tokens(self) -> int:
        return len(self.prompt) + len(self.output)

    @property
    def prefill_target(self) -> int:
        return len(self.prompt) if self.prefill_len is None else self.prefill_len

    @property
    def in_prefill(self) -> bool:
        return self.computed < self.prefill_target

    @property
    def done(self) -> bool:
        return self.status == SeqStatus.FINISHED


class TokenView:
    """Read-only concatenation of two token lists."""

    __slots__ = ("a", "b")

    def __init__(self, a: list[int], b: list[int]):
        self.a, self.b = a, b

    def __len__(self) -> int:
        return len(self.a) + len(self.b)

    def __iter__(self):
        yield from self.a
        yield from self.b

    def __eq__(self, other) -> bool:
        return list(self) == list(other)

    def __getitem__(self, i):
        na = len(self.a)
        if isinstance(i, slice):
            start, stop, step = i.indices(len(self))
            if step != 1:
                return list(self)[i]
            if stop <= na:
                return self.a[start:stop]
            if start >= na:
                return self.b[start - na:stop - na]
            return self.a[start:] + self.b[:stop - na]
        if i < 0:
            i += len(self)
        if not 0 <= i < len(self):
            raise IndexError("token index out of range")
        return self.a[i] if i < na else self.b[i - na]


@dataclasses.dataclass
class ScheduledChunk:
    seq: Sequence
    start: int        # first token position of this chunk
    num_tokens: int   # tokens fed this step
    is_prefill: bool
    needs_logits: bool


@dataclasses.dataclass
class SchedulerOutput:
    chunks: list[ScheduledChunk]
    num_tokens: int
    is_decode_only: bool
    preempted: list[Sequence] = dataclasses.field(default_factory=list)
    # decode rows and a prefill slice that run as two passes of one step (the
    # speculative decode graph covers decode rows only); see ``parts``
    split: bool = False

    def parts(self) -> tuple["SchedulerOutput", "SchedulerOutput"]:
        """The decode rows and the prefill chunks as separate outputs."""
        dec = [c for c in self.chunks if not c.is_prefill]
        pre = [c for c in self.chunks if c.is_prefill]
        return (SchedulerOutput(dec, sum(c.num_tokens for c in dec), True, self.preempted),
                SchedulerOutput(pre, sum(c.num_tokens for c in pre), False, []))


class Scheduler:
    def __init__(self, blocks: BlockManager, max_num_seqs: int = 4, max_num_batched_tokens: int = 4224,
                 decode_width: int = 1, max_model_len: int = 262144, lookahead: int = 0,
                 mix_prefill_with_decode: bool = True, prefill_slice: int = 0):
        if max_num_batched_tokens < 1 or max_num_seqs < 1:
            raise ValueError("scheduler limits must be positive")
        self.blocks = blocks
        self.max_num_seqs = max_num_seqs
        self.max_num_batched_tokens = max_num_batched_tokens
        self.decode_width = decode_width  # tokens per decoding sequence per step (1 + MTP drafts)
        self.max_model_len = max_model_len
        # KV slots a decoding sequence may write past its verify window (MTP drafts)
        self.lookahead = lookahead
        # False: decode rows and prefill chunks never share one forward (the
        # speculative step is one graph over decode rows only). With a
        # ``prefill_slice`` > 0 a step then carries the decode rows plus at
        # most that many prefill tokens, run as two passes (``split``), so a
        # long prompt delays each decode step by one slice only; with 0 steps
        # alternate between all-decode and all-prefill.
        self.mix = mix_prefill_with_decode
        if prefill_slice < 0:
            raise ValueError("prefill_slice must be >= 0")
        self.prefill_slice = int(prefill_slice)
        self._turn = 0
        self.waiting: collections.deque[Sequence] = collections.deque()
        self.running: list[Sequence] = []
        self._ids = itertools.count()
        self.num_preemptions = 0

    def add(self, prompt: list[int], params: SamplingParams | None = None) -> Sequence:
        if not prompt:
            raise ValueError("empty prompt")
        params = params or SamplingParams()
        if len(prompt) + params.max_tokens > self.max_model_len:
            raise ValueError("prompt + max_tokens exceeds max_model_len %d" % self.max_model_len)
        seq = Sequence(next(self._ids), list(prompt), params)
        self.waiting.append(seq)
        return seq

    def has_work(self) -> bool:
        return bool(self.waiting or self.running)

    def _admit(self, seq: Sequence) -> bool:
        """Admit the queue head if the pool holds its whole prefill. The blocks
        are reserved now, so the later chunks of a chunked prefill never find
        the pool emptied by decoding sequences in between."""
        try:
            # a request for prompt log-probabilities computes every prompt row: no prefix hits
            cached = self.blocks.allocate(seq.seq_id, seq.tokens[:seq.prefill_target],
                                          prefix=getattr(seq.params, "prompt_logprobs", None) is None)
        except CapacityError:
            return False
        try:
            self.blocks.ensure(seq.seq_id, seq.prefill_target)
        except CapacityError:  # allocate checked the same count; kept as a guard
            self.blocks.free_seq(seq.seq_id)
            return False
        seq.cached_tokens = cached
        seq.computed = cached
        seq.status = SeqStatus.RUNNING
        self.running.append(seq)
        return True

    def schedule(self) -> SchedulerOutput:
        budget = self.max_num_batched_tokens
        chunks: list[ScheduledChunk] = []
        preempted: list[Sequence] = []
        do_decode = do_prefill = True
        sliced = False
        if not self.mix:
            decoding = any(not s.in_prefill for s in self.running)
            prefilling = any(s.in_prefill for s in self.running) or (
                bool(self.waiting) and len(self.running) < self.max_num_seqs)
            if decoding and prefilling:
                if self.prefill_slice > 0:
                    sliced = True
                else:
                    self._turn ^= 1
                    do_decode, do_prefill = self._turn == 1, self._turn == 0
        # 1) decode tokens of generating sequences
        for seq in list(self.running) if do_decode else []:
            if seq.in_prefill:
                continue
            width = 1 + len(seq.draft)
            if width > budget:
                continue
            try:
                self.blocks.ensure(seq.seq_id, seq.computed + width + self.lookahead)
            except CapacityError:
                self._preempt(seq)
                preempted.append(seq)
                continue
            chunks.append(ScheduledChunk(seq, seq.computed, width, False, True))
            budget -= width
        if not do_prefill:
            return SchedulerOutput(chunks, sum(c.num_tokens for c in chunks), bool(chunks), preempted)
        if sliced and any(not c.is_prefill for c in chunks):
            budget = min(budget, self.prefill_slice)
        # 2) prefill chunks of admitted sequences, then admit new ones
        for seq in self.running:
            if budget <= 0:
                break
            if not seq.in_prefill or any(c.seq is seq for c in chunks):
                continue
            n = min(budget, seq.prefill_target - seq.computed)
            self.blocks.ensure(seq.seq_id, seq.computed + n)
            last = seq.computed + n == seq.prefill_target
            chunks.append(ScheduledChunk(seq, seq.computed, n, True, last))
            budget -= n
        while budget > 0 and self.waiting and len(self.running) < self.max_num_seqs:
            seq = self.waiting[0]
            if not self._admit(seq):
                break
            self.waiting.popleft()
            if seq.prefill_start is None:  # first admission (a preempted request keeps it)
                seq.prefill_start = time.monotonic()
            n = min(budget, seq.prefill_target - seq.computed)
            self.blocks.ensure(seq.seq_id, seq.computed + n)
            last = seq.computed + n == seq.prefill_target
            chunks.append(ScheduledChunk(seq, seq.computed, n, True, last))
            budget -= n
        total = sum(c.num_tokens for c in chunks)
        decode_only = bool(chunks) and all(not c.is_prefill for c in chunks)
        split = (not self.mix) and not decode_only and any(not c.is_prefill for c in chunks)
        return SchedulerOutput(chunks, total, decode_only, preempted, split)

    def _preempt(self, seq: Sequence) -> None:
        """Recompute-style preemption: free the blocks and requeue at the front.

        Prompt and output stay as they are (the output already streamed to the
        client, and ``max_tokens`` counts it); on readmission the sequence
        prefills every token it held and samples its next one from that
        prefill's last row."""
        self.blocks.free_seq(seq.seq_id)
        self.running.remove(seq)
        seq.status = SeqStatus.WAITING
        seq.prefill_len = seq.num_tokens
        seq.computed = 0
        seq.draft = []
        self.waiting.appendleft(seq)
        self.num_preemptions += 1

    def abort(self, seq_id: int) -> Sequence | None:
        """Finish a waiting or running sequence with reason ``abort``."""
        for seq in list(self.waiting) + list(self.running):
            if seq.seq_id == seq_id:
                if seq in self.waiting:
                    self.waiting.remove(seq)
                self.finish(seq, "abort")
                return seq
        return None

    def finish(self, seq: Sequence, reason: str) -> None:
        seq.status = SeqStatus.FINISHED
        seq.finish_reason = reason
        seq.finish_time = time.monotonic()
        if seq in self.running:
            self.running.remove(seq)
        self.blocks.free_seq(seq.seq_id)
