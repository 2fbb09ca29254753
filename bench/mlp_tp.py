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
  counter (decode sizes only: rows <= 64).

Activations are replicated (every rank holds all M rows), which is how the
engine's TP runs; the all-gather / reduce-scatter form is not built. Timed
with CUDA events over ``--iters`` layers after warm-up, max over ranks; an L2
flush (256 MB write) precedes every layer.

    python bench/mlp_tp.py                                   # TP1
    python -m torch.distributed.run --nproc-per-node N --master-addr 127.0.0.1 \\
        bench/mlp_tp.py [--comm nccl|fused] [--m 1,7,28,4224,16384]
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
    ap.add_argument("--m", default="1,7,28,4224,16384")
    ap.add_argument("--comm", default="nccl", choices=("nccl", "fused"))
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
    far = None
    if a.comm == "fused" and world > 1:
        from k8v4_xpu_b200.parallel.fused_ar import FusedAllReduce
        far = FusedAllReduce(None, torch.device("cuda", local), 64, H)
    down = _Shard(dq, ds)
    norm_w = torch.ones(H, dtype=torch.bfloat16, device="cuda")
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    results = []
    for M in [int(x) for x in a.m.split(",")]:
        xq = torch.randint(-127, 127, (M, H), dtype=torch.int8, device="cuda", generator=gen)
        xs = torch.rand(M, device="cuda", generator=gen) * 0.01
        gu = torch.empty(M, 2 * I // world, dtype=torch.bfloat16, device="cuda")
        out = torch.empty(M, H, dtype=torch.bfloat16, device="cuda")
        residual = torch.zeros(M, H, dtype=torch.bfloat16, device="cuda")
        fused = far is not None and far.fits(M, H)

        def layer():
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
        results.append({"M": M, "tp": world, "comm": "fused" if fused else "nccl", "layer_us": round(t * 1e6, 1),
                        "tflops_total": round(flops / t / 1e12, 1)})
    assert ops.status() == 0
    if rank == 0:
        print(json.dumps({"bench": "w4a8_mlp_tp", "gpus": world, "results": results}), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
