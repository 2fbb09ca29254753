#!/usr/bin/env python3
"""BASELINE config 2 at TP 1/2/4/8: the W4A8 MLP layer of the 27B decoder,
one process per GPU.

Each rank holds its shard: gate/up column-split (``2 * 17408 / tp`` output
features), down row-split (``17408 / tp`` input features). The layer is
gate_up -> SiLU-mul (+ int8 quant) -> down, whose partial output is summed
over the ranks and consumed by the next RMSNorm (+ residual):

* ``--comm nccl``: the GEMM writes bf16, then an NCCL all-reduce;
* ``--comm fused``: the down GEMM's epilogue adds fp32 partials into every
  rank's copy through NVLS multicast and the RMSNorm waits on the completion
  counter (decode sizes only: rows <= 64);
* ``--comm sp``: the prefill form (``parallel.seq_parallel``). The residual
  is sharded by 128-row token tiles; the down GEMM stores its bf16 partial
  rows straight into the owners' slots over NVLink (GEMM -> reduce-scatter),
  the owner's norm sums them and pushes its int8 rows to every rank through
  the multicast address, and the gate/up GEMM waits per owner tile for them
  (all-gather -> GEMM). Prefill sizes only (rows > 64, at most 16,384).

With ``nccl`` and ``fused`` the activations are replicated (every rank holds
all M rows). Timed with CUDA events over ``--iters`` layers after warm-up,
max over ranks; an L2 flush (256 MB write) precedes every layer. Each result
carries the layer's roofline: the slower of its per-rank MMA work at the
measured bf16 GEMM peak (the int8 tensor rate is twice that, nominally) and
the bytes that must cross NVLink per rank at 770 GB/s (the measured peer
copy rate per direction).

    python bench/mlp_tp.py                                   # TP1
    python -m torch.distributed.run --nproc-per-node N --master-addr 127.0.0.1 \\
        bench/mlp_tp.py [--comm nccl|fused|sp] [--rows 1,7,28,4224,16384]
"""
from __future__ import annotations

import argparse
import json
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import torch  # noqa: E402

from k8v4_xpu_b200 import ops  # noqa: E402
from k8v4_xpu_b200.parallel.comm import TPComm, init_from_env  # noqa: E402

H, I = 5120, 17408


def _peak():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        import json as _j
        return float(_j.load(open(p))["bf16_tflops"]), "measured bf16 GEMM burst"
    return 1590.0, "fallback bf16 GEMM burst"


TF, SRC = _peak()


def rand_int4(N, K, gen):
    qw = torch.randint(-2**31, 2**31 - 1, (K // 8, N), dtype=torch.int32, device="cuda", generator=gen)
    sc = (torch.rand(K // 128, N, device="cuda", generator=gen) * 0.01 + 0.001).half()
    return qw, sc


class _Shard:
    """Just enough of a linear for FusedAllReduce.gemm (weights + shape)."""

    def __init__(self, qweight, scales):
        self.qweight, self.scales = qweight, scales
        self.in_features, self.out_features = qweight.shape[0] * 8, qweight.shape[1]

    def split(self, rows, fused):
        return 1


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--rows", default="1,7,28,4224,16384", help="token rows (M) to run, comma separated")
    ap.add_argument("--comm", default="nccl", choices=("nccl", "fused", "sp"))
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    a = ap.parse_args()
    rank, world, local = init_from_env(timeout_s=300)
    torch.cuda.set_device(local)
    ops.require()
    comm = TPComm()
    if I % (world * 128):
        raise SystemExit("tp %d does not split the MLP on 128-wide groups" % world)
    gen = torch.Generator(device="cuda").manual_seed(1234 + rank)
    gq, gs = rand_int4(2 * I // world, H, gen)
    dq, ds = rand_int4(H, I // world, gen)
    far = sp = None
    if a.comm == "sp" and world > 1:
        from k8v4_xpu_b200.parallel.seq_parallel import SeqParallel
        sp = SeqParallel(None, torch.device("cuda", local), max(int(x) for x in a.rows.split(",")), H)
    if a.comm == "fused" and world > 1:
        from k8v4_xpu_b200.parallel.fused_ar import FusedAllReduce
        far = FusedAllReduce(None, torch.device("cuda", local), 64, H)
    down = _Shard(dq, ds)
    norm_w = torch.ones(H, dtype=torch.bfloat16, device="cuda")
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    results = []
    for M in [int(x) for x in a.rows.split(",")]:
        xq = torch.randint(-127, 127, (M, H), dtype=torch.int8, device="cuda", generator=gen)
        xs = torch.rand(M, device="cuda", generator=gen) * 0.01
        gu = torch.empty(M, 2 * I // world, dtype=torch.bfloat16, device="cuda")
        out = torch.empty(M, H, dtype=torch.bfloat16, device="cuda")
        residual = torch.zeros(M, H, dtype=torch.bfloat16, device="cuda")
        fused = far is not None and far.fits(M, H)
        use_sp = sp is not None and M > 64
        if use_sp:
            gate_up, down_l = _Shard(gq, gs), _Shard(dq, ds)
            sp.begin(M)
            x0 = torch.randn(max(1, sp.nrows), H, device="cuda", generator=gen).bfloat16()
            # the first norm starts the residual from local rows; every later
            # one sums the previous layer's reduce-scatter slots
            sp.norm_push(norm_w, 1e-6, gather=1, x_local=x0[: sp.nrows])

        def layer():
            if use_sp:
                gu_ = sp.gemm_ag(gate_up, 1)
                aq, as_ = ops.silu_mul(gu_, quant=True)
                sp.gemm_rs(down_l, 1, xq=aq, xs=as_)
                sp.norm_push(norm_w, 1e-6, gather=1, slot=1)
                return None
            ops.wq_gemm(ops.W4A8, gq, gs, xq, xscale=xs, out=gu)
            aq, as_ = ops.silu_mul(gu, quant=True)
            if fused:
                sums, sync = far.gemm(down, 1, xq=aq, xs=as_)
                return ops.rmsnorm(sums, norm_w, 1e-6, residual=residual, sync=sync)
            ops.wq_gemm(ops.W4A8, dq, ds, aq, xscale=as_, out=out)
            comm.all_reduce(out)
            return ops.rmsnorm(out, norm_w, 1e-6, residual=residual)

        for _ in range(a.warmup):
            layer()
        torch.cuda.synchronize()
        comm.barrier()
        total = 0.0
        for _ in range(a.iters):
            flush.fill_(1)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            layer()
            e1.record()
            e1.synchronize()
            total += e0.elapsed_time(e1) / 1e3
        torch.cuda.synchronize()
        comm.barrier()
        t = comm.max_scalar(total / a.iters)
        flops = 2 * M * 3 * I * H  # whole layer, all ranks
        mode = "sp" if use_sp else ("fused" if fused else "nccl")
        # bytes one rank must move over NVLink per layer (each direction):
        # its partial rows of the other ranks' tiles (bf16), and the other
        # ranks' normed rows (int8 + scale); replicated activations
        # (nccl / fused) all-reduce M x H bf16: 2 (world - 1) / world of it
        share = (world - 1) / world
        link = (M * H * 2 + M * (H + 4)) * share if use_sp else 2 * M * H * 2 * share
        t_mma = flops / world / (TF * 1e12)
        t_link = link / 770e9 if world > 1 else 0.0
        roof = max(t_mma, t_link)
        results.append({"M": M, "tp": world, "comm": mode, "layer_us": round(t * 1e6, 1),
                        "tflops_total": round(flops / t / 1e12, 1), "roofline_us": round(roof * 1e6, 1),
                        "bound": "mma" if t_mma >= t_link else "nvlink",
                        "frac_of_roofline": round(roof / t, 3), "peak_src": SRC})
    assert ops.status() == 0
    if rank == 0:
        print(json.dumps({"bench": "w4a8_mlp_tp", "gpus": world, "results": results}), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
