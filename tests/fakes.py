"""CPU stand-ins for GPU-only parts, used by the host-side tests."""
import time

from k8v4_xpu_b200.runtime.block_manager import BlockManager
from k8v4_xpu_b200.runtime.scheduler import Scheduler


class FakeEngine:
    """The engine's host contract (scheduler, block manager, stats, add/step/
    abort) with a deterministic 'model': the next token is last + 1."""

    def __init__(self, max_num_seqs=4, budget=64, block_size=16, num_blocks=256, max_model_len=4096, vocab=1000,
                 step_delay=0.0):
        self.blocks = BlockManager(num_blocks, block_size)
        self.scheduler = Scheduler(self.blocks, max_num_seqs, budget, 1, max_model_len)
        self.stats = {"steps": 0, "prompt_tokens": 0, "generated_tokens": 0, "iteration_tokens": []}
        self.mtp = None
        self.graphs = None
        self.vocab = vocab
        self.step_delay = step_delay

    def add_request(self, prompt, params=None):
        return self.scheduler.add(prompt, params)

    def has_unfinished(self):
        return self.scheduler.has_work()

    def abort(self, seq_id):
        self.scheduler.abort(seq_id)

    def step(self):
        out = self.scheduler.schedule()
        if self.step_delay:
            time.sleep(self.step_delay)
        finished = []
        now = time.monotonic()
        for c in out.chunks:
            seq = c.seq
            seq.computed = c.start + c.num_tokens
            if c.is_prefill:
                self.stats["prompt_tokens"] += c.num_tokens
            self.blocks.publish(seq.seq_id, seq.tokens, seq.computed)
            if not c.needs_logits:
                continue
            if getattr(seq.params, "prompt_logprobs", None) is not None and not seq.prompt_logprobs:
                seq.prompt_logprobs = [None] + [(-1.0, [])] * (len(seq.prompt) - 1)  # made up
            tok = (seq.tokens[-1] + 1) % self.vocab
            if seq.first_token_time is None:
                seq.first_token_time = now
            seq.output.append(tok)
            n_lp = getattr(seq.params, "logprobs", None)
            if n_lp is not None:  # a made-up distribution
                seq.logprobs.append((-0.5, [(tok, -0.5), (tok + 1, -1.5), (tok + 2, -2.5)][:n_lp]))
            self.stats["generated_tokens"] += 1
            p = seq.params
            if len(seq.output) >= p.max_tokens or (not p.ignore_eos and tok in p.stop_token_ids):
                self.scheduler.finish(seq, "length" if len(seq.output) >= p.max_tokens else "stop")
                finished.append(seq)
        self.stats["steps"] += 1
        self.stats["iteration_tokens"].append(out.num_tokens)
        return finished
