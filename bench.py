#!/usr/bin/env python3
"""Headline benchmark: decode tok/s at 128K context (c=1, c=4) and 128K prefill tok/s.

Model: the 27B-class dense K8/V4 decoder (64 layers, hidden 5120, 24 Q / 4 KV
heads, head_dim 128, vocab 151936, MLP 17408), random-init GPTQ INT4 weights,
INT8 embedding / lm_head, W4A8 MLP prefill, K8/V4 page-16 KV cache, tensor
parallel over N GPUs (one process per GPU, NCCL). Workload: a 128,197-token
uniform-random prompt prefilled in 4,224-token chunks, then decode at
concurrency 1 and 4 (the c=4 contexts are private copies of the prefilled
one, so each sequence reads its own KV pages every step).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

``value`` is decode tok/s at c=1 timed on the device (K back-to-back replays
of the captured decode step between CUDA events, max over ranks); ``e2e`` is
the same metric through the engine's public ``step()`` over 512 decode steps
(BASELINE config 3's decode length; ``--e2e-steps``), each one growing every
context by a token, with host scheduling, the H2D of the step inputs from
pinned memory and the D2H of the sampled tokens inside the timed region.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "decode tok/s @128K ctx (c=1,4) + prefill tok/s @128K, 27B W4A8 K8V4, 1-8 GPU"
BASE_DECODE = 78.02    # reference docs/w4a8-wiring-2026-10-02.md:27 (decode after fresh 128K prefill, c=1)
BASE_PREFILL = 1254.9  # reference docs/w4a8-wiring-2026-10-02.md:27 (fresh prefill @128,197)


def reference_arm() -> int:
    line = {"impl": "reference", "metric": METRIC,
            "unavailable": ("the reference (Wrapzii/k8v4-xpu) is a vLLM 0.30 patch whose kernels are SYCL/oneDNN "
                            "for Intel Xe2 XPUs; pip reports it 'not installable' (no setup.py/pyproject) and it "
                            "has no CUDA path, so it cannot run on a B200")}
    if int(os.environ.get("RANK", "0")) == 0:
        print(json.dumps(line), flush=True)
    return 0


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu: int):
        self.gpu = gpu
        self.proc = None
        self.lines: list[str] = []
        self.thread = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), "--query-gpu=" + self.FIELDS, "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (OSError, ValueError):
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        if self.thread:
            self.thread.join(timeout=2)
        return self.summarize(self.lines)

    @staticmethod
    def summarize(lines: list[str]) -> dict:
        """Median SM clock under load (power draw above 300 W; all samples if
        none), the max clock, and every throttle reason seen active."""
        sm, mx, reasons, loaded = [], None, set(), []
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for ln in lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
                if float(parts[3]) > 300.0:  # power.draw: the GPU is busy
                    loaded.append(float(parts[1]))
            except ValueError:
                continue
            for name, val in zip(names, parts[5:9]):
                if val.lower().startswith("active"):
                    reasons.add(name)
        use = sorted(loaded or sm)
        med = use[len(use) // 2] if use else None
        return {"sm_mhz": med, "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm),
                "samples_under_load": len(loaded)}


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=64)
    ap.add_argument("--warmup", type=int, default=4)
    ap.add_argument("--impl", default="ours", choices=("ours", "reference"))
    ap.add_argument("--ctx", type=int, default=128197)
    ap.add_argument("--chunk", type=int, default=4224)
    ap.add_argument("--model", default="dense-27b")
    ap.add_argument("--layers", type=int, default=None, help="debug only: fewer layers is not a valid number")
    ap.add_argument("--no-c4", action="store_true")
    ap.add_argument("--e2e-steps", type=int, default=512,
                    help="engine steps of the end-to-end decode (BASELINE config 3: 512 decode tokens)")
    ap.add_argument("--mode", default="decode", choices=("decode", "cp", "mtp"),
                    help="decode: the headline (128K prefill + decode c=1/c=4); cp: 262K context-parallel prefill "
                         "cold and cached-prefix TTFT; mtp: 4 x 200K contexts, MTP6 with forced acceptance 3.0")
    args = ap.parse_args()
    if args.impl == "reference":
        return reference_arm()
    if args.mode == "cp":
        return cp_mode(args)
    if args.mode == "mtp":
        return mtp_mode(args)
    args.warmup = max(3, args.warmup)

    import numpy as np
    import torch

    from k8v4_xpu_b200 import ops
    from k8v4_xpu_b200.models.config import PRESETS
    from k8v4_xpu_b200.parallel.comm import TPComm, init_from_env
    from k8v4_xpu_b200.runtime.engine import EngineConfig, LLMEngine
    from k8v4_xpu_b200.runtime.scheduler import SamplingParams

    rank, world, local = init_from_env(timeout_s=600)
    if world != args.gpus:
        raise SystemExit("launched with WORLD_SIZE=%d but --gpus %d" % (world, args.gpus))
    comm = TPComm()
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    ops.require()
    mcfg = PRESETS[args.model]
    ctx = args.ctx
    decode_budget = 2 * (args.warmup + args.steps + args.e2e_steps) + 64
    blocks_per_seq = (ctx + decode_budget + 15) // 16 + 2
    ecfg = EngineConfig(model=args.model, tensor_parallel_size=world, max_model_len=ctx + decode_budget + 16,
                        max_num_seqs=4, max_num_batched_tokens=args.chunk, num_kv_blocks=4 * blocks_per_seq + 8,
                        enable_prefix_caching=False, layers=args.layers, device=str(dev))
    t_init = time.perf_counter()
    eng = LLMEngine(ecfg, mcfg, comm=comm, rank=rank)
    torch.cuda.synchronize(dev)
    init_s = time.perf_counter() - t_init

    rng = np.random.default_rng(0)
    prompt = rng.integers(0, mcfg.vocab, size=ctx).tolist()
    params = SamplingParams(max_tokens=decode_budget, ignore_eos=True)

    def sync_all():
        torch.cuda.synchronize(dev)
        comm.barrier()

    # ---------------------------------------------------------------- prefill
    seq = eng.add_request(prompt, params)
    sync_all()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    w0 = time.perf_counter()
    e0.record()
    while not seq.output:
        eng.step()
    e1.record()
    sync_all()
    prefill_wall = comm.max_scalar(time.perf_counter() - w0)
    prefill_dev = comm.max_scalar(e0.elapsed_time(e1) / 1e3)

    # ----------------------------------------------------------------- decode
    def decode_phase(nseq: int) -> dict:
        # nvidia-smi needs ~1 s to start reporting: start it during the warm-up so
        # its samples cover the timed region (median over samples under load)
        sampler = ClockSampler(local)
        sampler.start()
        for _ in range(args.warmup):  # through the engine; captures graphs on first use
            eng.step()
        sync_all()
        graph = eng.graphs.graphs[(nseq, 1)][0]
        per_replay = eng.graphs.kernels[(nseq, 1)]
        for _ in range(3):
            graph.replay()
        sync_all()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(args.steps):
            graph.replay()
        b.record()
        sync_all()
        dev_s = comm.max_scalar(a.elapsed_time(b) / 1e3)
        # end to end: engine steps through the public API, each one advancing
        # every sequence by a token (the context grows; inputs go H2D from
        # pinned memory, the sampled tokens come back D2H)
        h2d0, d2h0 = eng.h2d_bytes, eng.d2h_bytes
        lens0 = [len(s_.prompt) + len(s_.output) for s_ in eng.scheduler.running]
        w = time.perf_counter()
        for _ in range(args.e2e_steps):
            eng.step()
        sync_all()
        e2e_s = comm.max_scalar(time.perf_counter() - w)
        lens1 = [len(s_.prompt) + len(s_.output) for s_ in eng.scheduler.running]
        clocks = sampler.stop()
        return {"dev_s": dev_s, "e2e_s": e2e_s, "clocks": clocks, "ctx": (min(lens0), max(lens1)),
                "h2d": (eng.h2d_bytes - h2d0) // args.e2e_steps, "d2h": (eng.d2h_bytes - d2h0) // args.e2e_steps,
                "launches": per_replay * args.steps}

    c1 = decode_phase(1)
    c4 = None
    if not args.no_c4:
        for _ in range(3):
            eng.clone_sequence_private(seq)
        sync_all()
        c4 = decode_phase(4)

    tok_c1 = args.steps / c1["dev_s"]
    line = {
        "metric": METRIC,
        "value": round(tok_c1, 2),
        "unit": "tok/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(1e3 * c1["dev_s"] / args.steps, 4),
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": round(tok_c1 / BASE_DECODE, 3),
        "dtype": "bf16",
        "data": "synthetic (uniform-random token prompt; random-init weights of the named architecture)",
        "config": {
            "model": "dense-27b: 64 layers, hidden 5120, 24q/4kv heads x 128, mlp 17408, vocab 151936; "
                     "GPTQ int4 g128 linears, int8 embedding + lm_head, W4A8 MLP prefill, K8/V4 page-16 KV",
            "global_batch": 1,
            "seq_len": ctx,
            "parallelism": "tp%d" % world,
            "prefill_chunk": args.chunk,
            "l2": "inputs larger than L2: each decode step reads ~10 GB of int4 weights and 6.6 GB of KV",
        },
        "prefill_tok_s": round(ctx / prefill_dev, 1),
        "prefill_s": round(prefill_dev, 3),
        "prefill_vs_baseline": round(ctx / prefill_dev / BASE_PREFILL, 3),
        "decode_c1_tok_s": round(tok_c1, 2),
        "clocks": c1["clocks"],
        "e2e": {
            "value": round(args.e2e_steps / c1["e2e_s"], 2),
            "unit": "tok/s",
            "steps": args.e2e_steps,
            "context": list(c1["ctx"]),
            "h2d_bytes_per_step": int(c1["h2d"]),
            "d2h_bytes_per_step": int(c1["d2h"]),
            "prefill_tok_s": round(ctx / prefill_wall, 1),
        },
        "gpu_launches": int(c1["launches"] + (c4["launches"] if c4 else 0)),
        "init_s": round(init_s, 1),
        "extension": ops.extension_path(),
    }
    if c4:
        line["decode_c4_tok_s"] = round(4 * args.steps / c4["dev_s"], 2)
        line["decode_c4_ms_per_step"] = round(1e3 * c4["dev_s"] / args.steps, 4)
        line["e2e"]["decode_c4_tok_s"] = round(4 * args.e2e_steps / c4["e2e_s"], 2)
        line["clocks_c4"] = c4["clocks"]
    if args.layers is not None or ctx != 128197:
        line["invalid"] = "debug run (layers=%s, ctx=%d)" % (args.layers, ctx)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if eng.graphs is not None:
        eng.graphs.release()
    comm.barrier()
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()
    return 0


def _emit(rank: int, line: dict) -> None:
    if rank == 0:
        print(json.dumps(line), flush=True)


def cp_mode(args) -> int:
    """262,144-token prefill with context parallelism over
    the ranks (KV pages sharded, peer pages read inside prefill attention),
    cold TTFT, then a request sharing the first 131,072 tokens (prefix hit)."""
    import numpy as np
    import torch

    from k8v4_xpu_b200.models.config import PRESETS
    from k8v4_xpu_b200.parallel.comm import TPComm, init_from_env
    from k8v4_xpu_b200.parallel.cp import CPGroup
    from k8v4_xpu_b200.runtime.cp_engine import CPEngine
    from k8v4_xpu_b200.runtime.engine import EngineConfig, LLMEngine
    from k8v4_xpu_b200.runtime.scheduler import SamplingParams
    rank, world, local = init_from_env(timeout_s=900)
    dev = torch.device("cuda", local)
    ctx = 262144 if args.ctx == 128197 else args.ctx
    shared = ctx // 2
    mcfg = PRESETS[args.model]
    blk = 16 * world
    blocks = 2 * ((ctx + 64 + blk - 1) // blk) + 8
    ecfg = EngineConfig(model=args.model, context_parallel_size=world, max_model_len=ctx + 64, max_num_seqs=2,
                        max_num_batched_tokens=args.chunk, num_kv_blocks=blocks, layers=args.layers,
                        device=str(dev), cuda_graphs=False)
    comm = TPComm()
    eng = CPEngine(ecfg, mcfg, CPGroup()) if world > 1 else LLMEngine(ecfg, mcfg)
    rng = np.random.default_rng(0)
    prompt = rng.integers(0, mcfg.vocab, size=ctx).tolist()
    second = prompt[:shared] + rng.integers(0, mcfg.vocab, size=ctx - shared).tolist()
    params = SamplingParams(max_tokens=1, ignore_eos=True)

    def ttft(p):
        torch.cuda.synchronize(dev)
        comm.barrier()
        seq = eng.add_request(p, params)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        w = time.perf_counter()
        a.record()
        while not seq.done:
            eng.step()
        b.record()
        torch.cuda.synchronize(dev)
        return comm.max_scalar(a.elapsed_time(b) / 1e3), comm.max_scalar(time.perf_counter() - w), seq

    cold_dev, cold_wall, s1 = ttft(prompt)
    hot_dev, hot_wall, s2 = ttft(second)
    line = {"metric": "context-parallel prefill TTFT @262K (cold, 131K cached prefix), 27B K8V4",
            "value": round(cold_dev, 3), "unit": "s", "higher_is_better": False, "n_gpus": world,
            "parallelism": "cp%d" % world, "ctx": ctx, "cold_ttft_s": round(cold_dev, 3),
            "cold_prefill_tok_s": round(ctx / cold_dev, 1), "cached_ttft_s": round(hot_dev, 3),
            "cached_prefix_tokens": s2.cached_tokens, "wall": {"cold_s": round(cold_wall, 3),
                                                               "cached_s": round(hot_wall, 3)},
            "dtype": "bf16", "data": "synthetic (uniform-random tokens; random-init weights)"}
    if args.layers is not None:
        line["invalid"] = "debug run (layers=%s)" % args.layers
    _emit(rank, line)
    comm.barrier()
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()
    return 0


def mtp_mode(args) -> int:
    """4 sequences holding 200,000-token contexts, MTP with 6
    drafts, 7-token verify under the speculative CUDA graph, acceptance forced
    to a seeded Bernoulli chain with mean accepted length 3.0."""
    import numpy as np
    import torch

    from k8v4_xpu_b200.models.config import PRESETS
    from k8v4_xpu_b200.parallel.comm import TPComm, init_from_env
    from k8v4_xpu_b200.runtime.engine import EngineConfig, LLMEngine
    from k8v4_xpu_b200.runtime.scheduler import SamplingParams
    rank, world, local = init_from_env(timeout_s=900)
    dev = torch.device("cuda", local)
    ctx = 200000 if args.ctx == 128197 else args.ctx
    mcfg = PRESETS[args.model]
    budget = 8 * (args.warmup + args.steps) + 64
    blocks_per_seq = (ctx + budget + 15) // 16 + 4
    comm = TPComm()
    ecfg = EngineConfig(model=args.model, tensor_parallel_size=world, max_model_len=ctx + budget + 16,
                        max_num_seqs=4, max_num_batched_tokens=args.chunk, num_kv_blocks=4 * blocks_per_seq + 8,
                        enable_prefix_caching=False, layers=args.layers, device=str(dev), speculative_tokens=6,
                        forced_accept_mean=3.0)
    eng = LLMEngine(ecfg, mcfg, comm=comm, rank=rank)
    rng = np.random.default_rng(0)
    seq = eng.add_request(rng.integers(0, mcfg.vocab, size=ctx).tolist(),
                          SamplingParams(max_tokens=budget, ignore_eos=True))
    while not seq.output:
        eng.step()
    for _ in range(3):
        eng.clone_sequence_private(seq)
    for _ in range(args.warmup):
        eng.step()
    torch.cuda.synchronize(dev)
    comm.barrier()
    gen0 = eng.stats["generated_tokens"]
    acc0 = (eng.mtp.stats.num_drafts, eng.mtp.stats.num_accepted_tokens)
    pos0 = list(eng.mtp.stats.accepted_per_pos)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(args.steps):
        eng.step()
    b.record()
    torch.cuda.synchronize(dev)
    dt = comm.max_scalar(a.elapsed_time(b) / 1e3)
    gen = eng.stats["generated_tokens"] - gen0
    nd = eng.mtp.stats.num_drafts - acc0[0]
    na = eng.mtp.stats.num_accepted_tokens - acc0[1]
    line = {"metric": "MTP6 decode tok/s, 4 x 200K contexts, forced acceptance mean 3.0, 27B K8V4",
            "value": round(gen / dt, 2), "unit": "tok/s", "higher_is_better": True, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(1e3 * dt / args.steps, 3),
            "mean_accepted_length": round(1 + na / max(1, nd), 3), "verify_rows": nd,
            "accepted_per_pos": [a - b for a, b in zip(eng.mtp.stats.accepted_per_pos, pos0)],
            "ctx": ctx, "concurrency": 4,
            "parallelism": "tp%d" % world, "timing": "engine steps (host scheduling included) between CUDA events",
            "dtype": "bf16", "data": "synthetic (uniform-random tokens; random-init weights)"}
    if args.layers is not None:
        line["invalid"] = "debug run (layers=%s)" % args.layers
    _emit(rank, line)
    eng.mtp.release()
    comm.barrier()
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
