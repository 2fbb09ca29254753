"""The serving engine: requests in, tokens out.

``LLMEngine`` owns one TP rank's model, its K8/V4 cache (one uint8 page
pool per layer; layers named in ``kv_cache_dtype_skip_layers`` get a plain
fp8 / bf16 pool on the same page ids, ``kv.skip_layers``), the block
manager, the scheduler, the decode CUDA-graph runner and the optional MTP
speculator. ``step()`` runs one scheduler step:

1. the scheduler picks decode tokens and prefill chunks (token budget 4,224);
2. the host builds the step's metadata (ids, positions, slots, block tables,
   lengths) in pinned memory and copies it to the device in one go;
3. decode-only steps replay a captured CUDA graph, other steps run eagerly;
4. the sampled ids come back to pinned host memory; sequences advance.

Every TP rank runs the same engine on the same request stream (rank 0 drives
the API; the others follow with identical scheduling decisions), so ranks
issue the same collectives in the same order. The reference runs stock
vLLM's engine with these settings (``k8v4_v030/launch.sh:176-194``: 4,224
batched tokens, prefix caching, MTP6, FULL_DECODE_ONLY graphs).
"""
from __future__ import annotations

import dataclasses
import os
import time

import numpy as np
import torch

from .. import ops
from ..kv import skip_layers
from ..models.config import ModelConfig
from ..models.dense import DenseModel, StepInputs
from . import sampling
from .block_manager import BlockManager, CapacityError
from .scheduler import SamplingParams, Scheduler, Sequence
from .workspace import Workspace

NUM_SMS = 148


@dataclasses.dataclass
class EngineConfig:
    """Typed engine configuration (CLI > env > defaults; see ``config.resolve``)."""

    model: str = "dense-27b"
    tensor_parallel_size: int = 1
    context_parallel_size: int = 1
    kv_cache_dtype: str = "int8_k_int4_v"
    max_model_len: int = 262144
    max_num_seqs: int = 4
    max_num_batched_tokens: int = 4224
    enable_prefix_caching: bool = True
    block_size: int = 16
    gpu_memory_utilization: float = 0.90
    num_kv_blocks: int | None = None
    speculative_tokens: int = 0      # MTP draft tokens per step (6 in the reference profile)
    cuda_graphs: bool = True          # FULL_DECODE_ONLY capture
    capture_sizes: tuple[int, ...] = ()
    seed: int = 0
    layers: int | None = None         # override (tests / smoke)
    forced_accept_mean: float | None = None  # MTP forced-acceptance benchmark mode
    # under MTP: prefill tokens that run beside each speculative decode step
    # while sequences decode (0: whole steps alternate between the two)
    mtp_prefill_slice: int = 1024
    device: str = "cuda"
    # layers whose KV stays in a plain dtype (the MTP layer's index is the
    # target's layer count); the dtype name is resolved from the environment
    # when None (K8V4_KV_SKIP_DTYPE, then VLLM_KV_SKIP_DTYPE, else auto)
    kv_cache_dtype_skip_layers: tuple[int, ...] = ()
    kv_skip_dtype: str | None = None

    def __post_init__(self):
        if self.kv_cache_dtype != "int8_k_int4_v":
            raise ValueError("kv_cache_dtype must be int8_k_int4_v")
        if self.max_num_batched_tokens < 1:
            raise ValueError("max_num_batched_tokens must be positive")
        self.kv_cache_dtype_skip_layers = skip_layers.parse_layers(self.kv_cache_dtype_skip_layers)
        if self.kv_cache_dtype_skip_layers or self.kv_skip_dtype is not None:
            self.kv_skip_dtype = skip_layers.resolve_skip_dtype(self.kv_skip_dtype)
        if self.kv_cache_dtype_skip_layers and self.context_parallel_size > 1:
            raise ValueError("skip layers are not supported under context parallelism")

    def skip_layouts(self, n_layers: int, hkv_local: int) -> dict[int, "skip_layers.SkipLayout"]:
        """Layer index -> plain-dtype cache layout; raises on an index outside
        the ``n_layers`` layers that hold a cache."""
        bad = [i for i in self.kv_cache_dtype_skip_layers if i >= n_layers]
        if bad:
            raise ValueError("skip layers %s outside the %d cached layers" % (bad, n_layers))
        return {i: skip_layers.SkipLayout(hkv_local, self.kv_skip_dtype) for i in self.kv_cache_dtype_skip_layers}


def decode_splits(max_pages: int, nseq: int, heads: int) -> int:
    """Split-K factor for decode attention: one full wave of CTAs.

    The kernel runs one CTA per SM, so splits * sequences * heads <= 148
    keeps every CTA in the first wave (a second partial wave measured
    slower than fewer, longer splits).
    """
    tiles = max(1, (max_pages + 7) // 8)
    want = max(1, NUM_SMS // max(1, nseq * heads))
    return int(max(1, min(want, tiles, 64)))


def stream_sync(device) -> None:
    """Wait for the device's current stream (host-side stand-in tensors on a
    CPU device need no wait)."""
    if torch.device(device).type == "cuda":
        torch.cuda.current_stream(device).synchronize()


class LLMEngine:
    def __init__(self, cfg: EngineConfig, model_cfg: ModelConfig, comm=None, rank: int = 0):
        self.cfg = cfg
        self.mcfg = model_cfg
        self.rank = rank
        self.tp = cfg.tensor_parallel_size
        self.device = torch.device(cfg.device)
        ops.require()
        self.model = DenseModel(model_cfg, tp=self.tp, rank=rank, device=self.device, comm=comm)
        self.model.random_init(seed=cfg.seed, layers=cfg.layers)
        if cfg.speculative_tokens:
            self.model.init_mtp(seed=cfg.seed)
        self.layout = self.model.layout
        self.tp_comm_mode = "single"
        if self.tp > 1:
            self._setup_tp_comm(comm)
        self._alloc_cache()
        self.blocks = BlockManager(self.num_blocks, cfg.block_size, self.layout.page, cfg.enable_prefix_caching)
        width = 1 + cfg.speculative_tokens
        spec = cfg.speculative_tokens > 0
        self.scheduler = Scheduler(self.blocks, cfg.max_num_seqs, cfg.max_num_batched_tokens, width,
                                   cfg.max_model_len, lookahead=width if spec else 0,
                                   mix_prefill_with_decode=not spec,
                                   prefill_slice=cfg.mtp_prefill_slice if spec else 0)
        # a decoding sequence may write up to 2 * width slots past its length (verify + drafts)
        self.max_pages = (cfg.max_model_len + 2 * width + self.layout.page - 1) // self.layout.page + 1
        self.max_q = max(1, width)
        self.max_tokens = max(cfg.max_num_batched_tokens, cfg.max_num_seqs * width)
        self.ws = Workspace(self.device, self.max_tokens, cfg.max_num_seqs, self.max_pages,
                            max(2 * model_cfg.intermediate // self.tp, model_cfg.hidden, 4096),
                            self.layout.hkv, self.layout.gqa, self.max_q, 64)
        self.graphs = None
        self.mtp = None
        if cfg.speculative_tokens:
            from ..spec.mtp import MTPSpeculator
            self.mtp = MTPSpeculator(self, cfg.speculative_tokens, cfg.forced_accept_mean, cfg.seed)
        if cfg.cuda_graphs and self.mtp is None:
            from .graphs import DecodeGraphs
            self.graphs = DecodeGraphs(self)
        # pinned host staging for the per-step copies
        self._pin_i64 = torch.zeros(4 * self.max_tokens, dtype=torch.int64, pin_memory=True)
        self._pin_i32 = torch.zeros(2 * (cfg.max_num_seqs + 1) + cfg.max_num_seqs * self.max_pages
                                    + self.max_tokens, dtype=torch.int32, pin_memory=True)
        self._pin_out = torch.zeros(self.max_tokens, dtype=torch.int64, pin_memory=True)
        self.h2d_bytes = 0
        self.d2h_bytes = 0
        self._h2d_done = None
        self.stats = {"steps": 0, "prompt_tokens": 0, "generated_tokens": 0, "prefill_time": 0.0,
                      "decode_time": 0.0, "iteration_tokens": []}

    def _setup_tp_comm(self, comm) -> None:
        """Fused GEMM -> all-reduce (NVLS multicast) for decode-sized steps
        when the box supports it; NCCL otherwise and for larger steps."""
        from ..parallel.fused_ar import FusedAllReduce, fused_ar_mode
        self.tp_comm_mode = "nccl"
        self.tp_prefill_mode = "nccl"
        if fused_ar_mode() != "fused":
            return
        rows = max(self.cfg.max_num_seqs * (1 + self.cfg.speculative_tokens), 1)
        rows = min(64, max(rows, 8))
        try:
            self.model.fused_ar = FusedAllReduce(getattr(comm, "group", None), self.device, rows,
                                                 self.mcfg.hidden)
            self.tp_comm_mode = "fused"
        except Exception as e:  # no multicast on this box: NCCL all-reduce
            import logging
            logging.getLogger("k8v4").warning("fused all-reduce unavailable (%s); using NCCL", e)
        # prefill chunks, with K8V4_TP_PREFILL=sp (the default is GEMM + NCCL):
        # sequence parallelism with the reduce-scatter and the all-gather fused
        # into the GEMMs
        from ..parallel.seq_parallel import SeqParallel, sp_mode
        self.tp_prefill_mode = "nccl"
        if sp_mode() != "sp":
            return
        try:
            self.model.sp = SeqParallel(getattr(comm, "group", None), self.device, self.cfg.max_num_batched_tokens,
                                        self.mcfg.hidden)
            self.tp_prefill_mode = "sp"
        except Exception as e:  # no multicast on this box: NCCL all-reduce
            import logging
            logging.getLogger("k8v4").warning("sequence-parallel prefill unavailable (%s); using NCCL", e)

    # ---------------------------------------------------------------- cache
    def _alloc_cache(self) -> None:
        cfg = self.cfg
        page_bytes = self.layout.page_bytes
        # the MTP draft layer keeps its own cache after the target's layers
        n_layers = len(self.model.layers) + (1 if self.model.mtp is not None else 0)
        skip = cfg.skip_layouts(n_layers, self.model.shape.hkv_local)
        per_page = skip_layers.pool_bytes_per_page(page_bytes, n_layers, skip)
        if cfg.num_kv_blocks is not None:
            blocks = int(cfg.num_kv_blocks)
        else:
            free, total = torch.cuda.mem_get_info(self.device)
            budget = free - (1 - cfg.gpu_memory_utilization) * total - (4 << 30)
            blocks = int(budget // (per_page * (cfg.block_size // self.layout.page)))
            need = ((cfg.max_model_len + cfg.block_size - 1) // cfg.block_size + 1) * cfg.max_num_seqs
            blocks = max(1, min(blocks, need))
        if blocks < 1:
            raise CapacityError("no memory left for the KV cache", fit_tokens=0)
        if blocks * cfg.block_size < cfg.max_model_len:
            fit = blocks * cfg.block_size - 2 * (1 + cfg.speculative_tokens)
            raise CapacityError("max_model_len %d exceeds the KV cache capacity of %d tokens"
                                % (cfg.max_model_len, blocks * cfg.block_size), fit_tokens=max(0, fit))
        self.num_blocks = blocks
        pages = blocks * (cfg.block_size // self.layout.page)
        self.kv_pool = torch.empty((n_layers - len(skip), pages, page_bytes), dtype=torch.uint8, device=self.device)
        dense = iter(range(n_layers - len(skip)))
        self.kv_caches = [skip[i].alloc(pages, self.device) if i in skip else self.kv_pool[next(dense)]
                          for i in range(n_layers)]
        self.model.skip_kv = skip
        self.kv_capacity_tokens = blocks * cfg.block_size
        import logging
        logging.getLogger("k8v4").info(
            "KV cache size: %d tokens (%d blocks of %d, %.2f GiB over %d layers%s)", self.kv_capacity_tokens, blocks,
            cfg.block_size, pages * per_page / 2 ** 30, n_layers,
            ", skip layers %s in %s" % (sorted(skip), cfg.kv_skip_dtype) if skip else "")

    # ------------------------------------------------------------- requests
    def add_request(self, prompt: list[int], params: SamplingParams | None = None) -> Sequence:
        if params is not None:
            if params.temperature < 0 or not 0.0 < params.top_p <= 1.0 or params.top_k < 0:
                raise ValueError("temperature must be >= 0, top_p in (0, 1], top_k >= 0")
            if params.logprobs is not None and not 0 <= params.logprobs <= 20:
                raise ValueError("logprobs must lie in [0, 20]")
            if params.repetition_penalty <= 0 or not -2.0 <= params.presence_penalty <= 2.0 \
                    or not -2.0 <= params.frequency_penalty <= 2.0:
                raise ValueError("repetition_penalty must be > 0; presence / frequency penalties in [-2, 2]")
            if params.prompt_logprobs is not None:
                if not 0 <= params.prompt_logprobs <= 20:
                    raise ValueError("prompt_logprobs must lie in [0, 20]")
                if getattr(self, "cp", None) is not None:
                    raise ValueError("prompt log-probabilities are not served under context parallelism")
        return self.scheduler.add(prompt, params)

    def has_unfinished(self) -> bool:
        return self.scheduler.has_work()

    def abort(self, seq_id: int) -> None:
        self.scheduler.abort(seq_id)

    # ----------------------------------------------------------------- step
    def _build_inputs(self, sched) -> tuple[StepInputs, list]:
        """Pack the step's metadata on the host, copy it to the device once."""
        chunks = sched.chunks
        T = sched.num_tokens
        B = len(chunks)
        ids = np.zeros(T, np.int64)
        pos = np.zeros(T, np.int64)
        slots = np.zeros(T, np.int64)
        cu = np.zeros(B + 1, np.int32)
        lens = np.zeros(B, np.int32)
        logit_rows = []
        tables = []
        t = 0
        max_q = 1
        for i, c in enumerate(chunks):
            seq = c.seq
            toks = seq.tokens
            n = c.num_tokens
            feed = toks[c.start:c.start + n] if c.is_prefill else ([toks[-1]] + seq.draft)[:n]
            ids[t:t + n] = feed
            pos[t:t + n] = np.arange(c.start, c.start + n)
            for j in range(n):
                slots[t + j] = self.blocks.slot(seq.seq_id, c.start + j)
            cu[i + 1] = t + n
            lens[i] = c.start + n
            if c.needs_logits:
                if c.is_prefill:
                    logit_rows.append(t + n - 1)
                else:
                    logit_rows.extend(range(t, t + n))
            tables.append(self.blocks.page_table(seq.seq_id))
            max_q = max(max_q, n)
            t += n
        W = max(len(tb) for tb in tables)
        bt = np.zeros((B, W), np.int32)
        for i, tb in enumerate(tables):
            bt[i, :len(tb)] = tb
        dev = self.device
        # the previous step's async copies must have drained the pinned buffers
        if self._h2d_done is not None:
            self._h2d_done.synchronize()
        # one pinned staging buffer per dtype, one async copy each
        L = len(logit_rows)
        i64 = self._pin_i64[: 3 * T + L].numpy()
        i64[:T], i64[T:2 * T], i64[2 * T:3 * T], i64[3 * T:] = ids, pos, slots, logit_rows
        i32 = self._pin_i32[: B + 1 + B + B * W].numpy()
        i32[: B + 1] = cu
        i32[B + 1: 2 * B + 1] = lens
        i32[2 * B + 1:] = bt.reshape(-1)
        # copy=True: the inputs never alias the staging buffer (they would on a CPU device)
        g64 = self._pin_i64[: 3 * T + L].to(dev, non_blocking=True, copy=True)
        g32 = self._pin_i32[: 2 * B + 1 + B * W].to(dev, non_blocking=True, copy=True)
        self.h2d_bytes += g64.numel() * 8 + g32.numel() * 4
        if dev.type == "cuda":
            self._h2d_done = torch.cuda.Event()
            self._h2d_done.record(torch.cuda.current_stream(dev))
        inp = StepInputs(
            input_ids=g64[:T], positions=g64[T:2 * T], slots=g64[2 * T:3 * T], logit_rows=g64[3 * T:],
            cu_q=g32[: B + 1], seq_lens=g32[B + 1: 2 * B + 1], block_table=g32[2 * B + 1:].view(B, W),
            max_q_len=max_q, is_decode=sched.is_decode_only and max_q * self.layout.gqa <= 64,
        )
        if inp.is_decode:
            # same split count as the captured graphs: eager and graph decode are bitwise equal
            inp.nsplit = decode_splits(self.max_pages, B, self.layout.hkv)
        return inp, logit_rows

    def step(self) -> list[Sequence]:
        """One scheduler step. Returns sequences that finished during it."""
        sched = self.scheduler.schedule()
        if not sched.chunks:
            return []
        t0 = time.perf_counter()
        if self.mtp is not None and sched.split:
            # the speculative graph over the decode rows, then the prefill slice
            dec, pre = sched.parts()
            finished = self.mtp.step(dec) + self._plain_step(pre)
        elif self.mtp is not None and sched.is_decode_only:
            finished = self.mtp.step(sched)
        else:
            finished = self._plain_step(sched)
        dt = time.perf_counter() - t0
        self.stats["steps"] += 1
        its = self.stats["iteration_tokens"]  # the metrics exporter drains it
        its.append(sched.num_tokens)
        if len(its) > 65536:  # nothing drains it: keep the recent half
            del its[:32768]
        if sched.is_decode_only:
            self.stats["decode_time"] += dt
        else:
            self.stats["prefill_time"] += dt
        return finished

    def _plain_step(self, sched) -> list[Sequence]:
        if self.graphs is not None and sched.is_decode_only and self.graphs.can_run(sched):
            tokens = self.graphs.run(sched)
        elif self.mtp is not None:
            # speculative serving: the MTP layer catches up on every prefill row
            inp, rows = self._build_inputs(sched)
            hid_all = self.model.forward(inp, self.kv_caches, self.ws, all_rows=True)
            seqs = [c.seq for c in sched.chunks if c.needs_logits]
            self._prompt_logprobs(sched, hid_all)
            tokens = self._sample(hid_all.index_select(0, inp.logit_rows), seqs) if rows else np.zeros(0, np.int64)
            self.mtp.after_prefill(sched, inp, hid_all, tokens)
        else:
            inp, rows = self._build_inputs(sched)
            if any(c.is_prefill and sampling.wants_prompt_logprobs(c.seq.params) for c in sched.chunks):
                hid_all = self.model.forward(inp, self.kv_caches, self.ws, all_rows=True)
                self._prompt_logprobs(sched, hid_all)
                hidden = hid_all.index_select(0, inp.logit_rows)
            else:
                hidden = self.model.forward(inp, self.kv_caches, self.ws)
            # a step made only of non-final prefill chunks samples nothing
            seqs = [c.seq for c in sched.chunks if c.needs_logits]
            tokens = self._sample(hidden, seqs) if rows else np.zeros(0, np.int64)
        return self._commit(sched, tokens)

    def _prompt_logprobs(self, sched, hid_all: torch.Tensor, rows_per_call: int = 256) -> None:
        """Log-probabilities of the prompt tokens in this step's prefill chunks,
        for the requests that ask for them: row p of a chunk scores the prompt
        token at p + 1 (``seq.prompt_logprobs[k]`` is prompt token k's entry;
        the first token has none). Logits are made ``rows_per_call`` rows at a
        time (under TP every rank gathers the vocabulary shards alike)."""
        t = 0
        for c in sched.chunks:
            seq, n = c.seq, c.num_tokens
            if c.is_prefill and sampling.wants_prompt_logprobs(seq.params):
                if c.start == 0 and not seq.prompt_logprobs:
                    seq.prompt_logprobs.append(None)
                rows, targets = [], []
                for j in range(n):
                    p = c.start + j
                    if p + 1 < len(seq.prompt) and p + 1 == len(seq.prompt_logprobs) + len(targets):
                        rows.append(t + j)
                        targets.append(seq.prompt[p + 1])
                for k in range(0, len(rows), rows_per_call):
                    idx = torch.tensor(rows[k:k + rows_per_call], dtype=torch.int64, device=self.device)
                    lg = self.model.logits(hid_all.index_select(0, idx))
                    if self.tp > 1:
                        lg = self.model.comm.all_gather(lg, dim=1)
                    seq.prompt_logprobs.extend(
                        sampling.logprob_rows(lg, targets[k:k + rows_per_call], seq.params.prompt_logprobs))
            t += n

    def _choose(self, hidden: torch.Tensor, seqs: list[Sequence] | None = None) -> torch.Tensor:
        """Next-token ids [rows] on the device: the argmax kernel, or, when a
        row's request samples, asks for log-probabilities or sets penalties,
        the full-vocabulary logits (the TP shards gathered on every rank),
        penalized, then the argmax or a seeded draw; log-probability entries
        wait in the engine's stash for the commit (``runtime.sampling``)."""
        if not seqs or not any(sampling.needs_logits(s.params) for s in seqs):
            return self.model.greedy(hidden)
        lg = self.model.logits(hidden)
        if self.tp > 1:
            lg = self.model.comm.all_gather(lg, dim=1)
        gens = [sampling.generator_for(s, self.cfg.seed, self.device) if sampling.samples(s.params) else None
                for s in seqs]
        pick = lg
        if any(sampling.has_processors(s.params) for s in seqs):
            pick = lg.float().clone()
            for i, s in enumerate(seqs):
                if sampling.has_processors(s.params):
                    pick[i] = sampling.process_row(lg[i], s.prompt, s.output, s.params, holder=s)
        ids = sampling.sample_rows(pick, [s.params for s in seqs], gens)
        if any(sampling.wants_logprobs(s.params) for s in seqs):
            host = ids.tolist()
            stash = sampling.stash_of(self)
            for i, s in enumerate(seqs):
                if sampling.wants_logprobs(s.params):
                    stash[s.seq_id] = [sampling.logprob_entry(lg[i], host[i], s.params.logprobs)]
        return ids

    def _agree(self, ids: torch.Tensor) -> torch.Tensor:
        """Hook for engines whose ranks sample replicated rows (context
        parallelism): makes every rank hold the same ids."""
        return ids

    def _sample(self, hidden: torch.Tensor, seqs: list[Sequence] | None = None) -> np.ndarray:
        ids = self._agree(self._choose(hidden, seqs))
        n = ids.numel()
        out = self._pin_out[:n]
        out.copy_(ids, non_blocking=True)
        stream_sync(self.device)
        self.d2h_bytes += n * 8
        return out.numpy().copy()

    def _commit(self, sched, tokens: np.ndarray) -> list[Sequence]:
        finished = []
        k = 0
        now = time.monotonic()
        for c in sched.chunks:
            seq = c.seq
            seq.computed = c.start + c.num_tokens
            if c.is_prefill:
                self.stats["prompt_tokens"] += c.num_tokens
            self.blocks.publish(seq.seq_id, seq.tokens, seq.computed)
            if not c.needs_logits:
                continue
            tok = int(tokens[k])
            k += 1
            if seq.first_token_time is None:
                seq.first_token_time = now
            seq.output.append(tok)
            sampling.record(self, seq)
            self.stats["generated_tokens"] += 1
            if self._should_stop(seq, tok):
                self.scheduler.finish(seq, "length" if len(seq.output) >= seq.params.max_tokens else "stop")
                finished.append(seq)
        return finished

    def _should_stop(self, seq: Sequence, tok: int) -> bool:
        if len(seq.output) >= seq.params.max_tokens:
            return True
        if seq.params.allowed_sequences and sampling.choice_finished(seq.params, seq.output):
            return True
        return (not seq.params.ignore_eos) and tok in seq.params.stop_token_ids

    # ------------------------------------------------------------ helpers
    def generate(self, prompts: list[list[int]], params: SamplingParams | None = None) -> list[list[int]]:
        seqs = [self.add_request(p, params) for p in prompts]
        while self.has_unfinished():
            self.step()
        return [s.output for s in seqs]

    def fork_sequence(self, seq: Sequence) -> Sequence:
        """A new running sequence with the same tokens and its own copy of the KV tail."""
        child = Sequence(next(self.scheduler._ids), list(seq.prompt), seq.params, list(seq.output),
                         prefill_len=seq.prefill_len)
        copies = self.blocks.fork(seq.seq_id, child.seq_id, seq.computed)
        r = self.blocks.ratio
        for src, dst in copies:
            for layer in self.kv_caches:
                layer[dst * r:(dst + 1) * r].copy_(layer[src * r:(src + 1) * r])
        child.computed = seq.computed
        child.status = seq.status
        child.first_token_time = seq.first_token_time
        self.scheduler.running.append(child)
        return child

    def clone_sequence_private(self, seq: Sequence) -> Sequence:
        """A new running sequence holding a private copy of every KV page.

        Used to build several long contexts from one prefill without sharing
        pages (so concurrent decodes read distinct memory).
        """
        child = Sequence(next(self.scheduler._ids), list(seq.prompt), seq.params, list(seq.output),
                         prefill_len=seq.prefill_len)
        child.draft = list(seq.draft)
        self.blocks.tables[child.seq_id] = []
        self.blocks.keys[child.seq_id] = []
        self.blocks.ensure(child.seq_id, seq.computed)
        n = (seq.computed + self.layout.page - 1) // self.layout.page  # pages with written KV
        src = torch.tensor(self.blocks.page_table(seq.seq_id)[:n], device=self.device)
        dst = torch.tensor(self.blocks.page_table(child.seq_id)[:n], device=self.device)
        for layer in self.kv_caches:
            layer.index_copy_(0, dst, layer.index_select(0, src))
        child.computed = seq.computed
        child.status = seq.status
        child.first_token_time = seq.first_token_time
        self.scheduler.running.append(child)
        return child
