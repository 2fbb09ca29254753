"""Row-parallel GEMM + all-reduce + RMSNorm at decode sizes: NCCL vs fused.

    torchrun --nproc-per-node N bench/tp_allreduce_micro.py [--rows 1 4 7 28]

For the o_proj (K = 3072 / tp) and down_proj (K = 17408 / tp) shapes of the
27B decoder (N = hidden = 5120), times ``--iters`` back-to-back
(GEMM -> all-reduce -> residual + RMSNorm) sequences captured in one CUDA
graph, on each rank with CUDA events, and prints the max over ranks:

* ``nccl``  : split-K GEMM + finish -> NCCL all-reduce (bf16) -> RMSNorm;
* ``fused`` : GEMM with multimem.red epilogue into the NVLS multicast buffer
  -> RMSNorm that waits on the completion counter.

Roofline per call: max(weight bytes / HBM bandwidth, NVLink bytes / 770 GB/s),
NVLink bytes = split x rows x N x 4 (the fp32 partials each rank pushes).
"""
from __future__ import annotations

import argparse
import json
import os
import sys

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--rows", type=int, nargs="+", default=[1, 4, 7, 28])
    ap.add_argument("--iters", type=int, default=64)
    args = ap.parse_args()
    from k8v4_xpu_b200 import ops
    from k8v4_xpu_b200.layers.linear import Int4Linear
    from k8v4_xpu_b200.models import gptq
    from k8v4_xpu_b200.parallel.comm import TPComm, init_from_env
    from k8v4_xpu_b200.parallel.fused_ar import FusedAllReduce

    rank, world, local = init_from_env(timeout_s=300)
    dev = torch.device("cuda", local)
    comm = TPComm()
    H = 5120
    peaks = {}
    pk = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "MEASURED_PEAKS.json")
    if os.path.exists(pk):
        peaks = json.load(open(pk))
    hbm = float(peaks.get("hbm_gbs", 6650.0)) * 1e9
    far = FusedAllReduce(None, dev, 64, H)
    g = torch.Generator(device=dev).manual_seed(0)
    results = []
    for name, K in (("o_proj", 3072 // world), ("down_proj", 17408 // world)):
        w = torch.randn(K, H, generator=g, device=dev) * 0.02
        codes, sc = gptq.quantize_int4_rtn(w)
        pw = gptq.pack_int4(codes, sc)
        lin = Int4Linear(name, pw["qweight"], pw["scales"])
        norm_w = torch.ones(H, dtype=torch.bfloat16, device=dev)
        for M in args.rows:
            x = torch.randn(M, K, generator=g, device=dev).bfloat16()
            res = torch.randn(M, H, generator=g, device=dev).bfloat16()
            ws = torch.zeros(64 * H, dtype=torch.float32, device=dev)
            split = lin.split(M, ws)

            def nccl_body():
                y = lin(x, ws=ws, split=split)
                comm.all_reduce(y)
                return ops.rmsnorm(y, norm_w, 1e-6, residual=res)

            def fused_body():
                y, sync = far.gemm(lin, 0, x=x)
                return ops.rmsnorm(y, norm_w, 1e-6, residual=res, sync=sync)

            row = {"gemm": name, "rows": M, "K": K, "N": H, "split": split, "world": world}
            for tag, body in (("nccl", nccl_body), ("fused", fused_body)):
                s = torch.cuda.Stream(device=dev)
                s.wait_stream(torch.cuda.current_stream(dev))
                with torch.cuda.stream(s):
                    for _ in range(3):
                        body()
                torch.cuda.current_stream(dev).wait_stream(s)
                graph = torch.cuda.CUDAGraph()
                with torch.cuda.graph(graph, stream=s):
                    for _ in range(args.iters):
                        body()
                for _ in range(2):
                    graph.replay()
                torch.cuda.synchronize(dev)
                comm.barrier()
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record()
                graph.replay()
                b.record()
                torch.cuda.synchronize(dev)
                us = comm.max_scalar(a.elapsed_time(b) * 1e3 / args.iters)
                row[tag + "_us"] = round(us, 2)
                del graph
            wbytes = K * H / 2 + (K // 128) * H * 2
            nv = split * M * H * 4
            roof_us = max(wbytes / hbm, nv / 770e9) * 1e6
            row["roofline_us"] = round(roof_us, 2)
            row["fused_frac_of_roofline"] = round(roof_us / row["fused_us"], 3)
            row["nccl_frac_of_roofline"] = round(roof_us / row["nccl_us"], 3)
            results.append(row)
            if rank == 0:
                print(json.dumps(row), flush=True)
    st = ops.status()
    comm.barrier()
    if rank == 0:
        print(json.dumps({"status": st}), flush=True)
    dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
