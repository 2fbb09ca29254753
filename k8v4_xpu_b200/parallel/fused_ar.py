"""GEMM -> all-reduce fused over NVLink SHARP (NVLS multicast) for TP decode.

The row-parallel projections of a TP layer (o_proj and the MLP down_proj)
end in an all-reduce of their ``[T, hidden]`` output. The reference did that
with a separate oneCCL all-reduce after each GEMM (vLLM's TP, tuned in
``k8v4_v030/launch.sh:101-110``). Here the GEMM's epilogue does it:

* each rank's fp32 partial sums go out with ``multimem.red.add.f32`` to the
  multicast address of a symmetric buffer, so the NVSwitch adds them into
  every rank's copy while the GEMM's other tiles are still in flight;
* each CTA then adds 1 to a multicast completion counter (release, system
  scope);
* the RMSNorm that consumes the sum (plus the residual add, the norm, and the
  W4A8 int8 quantization when it applies) waits until its local copy of the
  counter has every rank's CTAs, reads the sums from its own copy and zeroes
  them for the next use.

Two buffers alternate (o_proj uses slot 0, down_proj slot 1): a rank can
only start writing a slot again after every rank passed the other slot's
counter, which every rank reaches after consuming this one.

Torch's symmetric memory does the plumbing (allocation, handle exchange,
multicast object); the kernels issue the multimem operations themselves.

Each rank's copy receives world x the partial's bytes (every rank's adds
land in every copy), so the path serves decode-sized GEMMs (at most
``max_rows`` rows); larger calls keep the NCCL all-reduce.
"""
from __future__ import annotations

import os

import torch
import torch.distributed as dist

from .. import ops


def fused_ar_mode() -> str:
    """``K8V4_TP_COMM`` = ``fused`` (default: multimem GEMM epilogue where the
    box supports multicast) or ``nccl`` (GEMM, then an NCCL all-reduce)."""
    mode = os.environ.get("K8V4_TP_COMM", "fused").strip().lower()
    if mode not in ("fused", "nccl"):
        raise ValueError("K8V4_TP_COMM must be fused or nccl, got %r" % mode)
    return mode


def gemv_fused() -> bool:
    """``K8V4_TP_GEMV_FUSED=1``: one-row row-parallel GEMMs use the decode
    GEMV's multicast all-reduce epilogue instead of GEMV + NCCL."""
    return os.environ.get("K8V4_TP_GEMV_FUSED", "0").strip().lower() in ("1", "true", "yes")


class FusedAllReduce:
    SLOTS = 2

    def __init__(self, group, device: torch.device, max_rows: int, hidden: int):
        import torch.distributed._symmetric_memory as symm_mem
        self.group = group if group is not None else dist.group.WORLD
        self.world = dist.get_world_size(self.group)
        self.rank = dist.get_rank(self.group)
        self.device = torch.device(device)
        self.max_rows = int(max_rows)
        self.hidden = int(hidden)
        per = self.max_rows * self.hidden
        self.data = symm_mem.empty(self.SLOTS * per, dtype=torch.float32, device=self.device)
        self.flags = symm_mem.empty(16, dtype=torch.int64, device=self.device)
        self.data.zero_()
        self.flags.zero_()
        hd = symm_mem.rendezvous(self.data, self.group.group_name)
        hf = symm_mem.rendezvous(self.flags, self.group.group_name)
        if not (hd.has_multicast_support and hf.has_multicast_support):
            raise RuntimeError("symmetric memory on this box has no multicast (NVLS) support")
        self._handles = (hd, hf)
        self.data_mc = int(hd.multicast_ptr)
        self.flag_mc = int(hf.multicast_ptr)
        if self.data_mc == 0 or self.flag_mc == 0:
            raise RuntimeError("no multicast address for the all-reduce buffers")
        if self.data_mc == self.data.data_ptr() or self.flag_mc == self.flags.data_ptr():
            # multimem instructions need a real multicast mapping, not the unicast buffer
            raise RuntimeError("the multicast address is the local buffer (no multicast object)")
        # per slot: [signals consumed so far, consumer CTAs done] (local to this rank)
        self.state = torch.zeros((self.SLOTS, 2), dtype=torch.int64, device=self.device)
        # one-row calls (the decode GEMV): per slot a local fp32 row where the
        # partial sums meet before one CTA sends them, and that CTA's ticket
        self.gemv_local = torch.zeros((self.SLOTS, ops.GEMV_MAX_ROWS * self.hidden), dtype=torch.float32,
                                      device=self.device)
        self.gemv_ticket = torch.zeros((self.SLOTS, 4), dtype=torch.int32, device=self.device)
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)  # every copy is zero before the first multicast add
        self.calls = 0

    def fits(self, rows: int, n: int) -> bool:
        """Calls this path serves. One-row calls run as the decode GEMV; there
        the GEMV followed by an NCCL all-reduce measured faster (TP2, 128K,
        c = 1: 172.2 tok/s against 161.9 with the GEMV's own multicast
        epilogue), so they take NCCL unless ``K8V4_TP_GEMV_FUSED=1``."""
        if rows == 1 and ops.takes_gemv(ops.W4A16, 1, True) and not gemv_fused():
            return False
        return 0 < rows <= self.max_rows and n == self.hidden

    def gemm(self, linear, slot: int, x: torch.Tensor | None = None, xq: torch.Tensor | None = None,
             xs: torch.Tensor | None = None, split: int | None = None):
        """Run ``linear`` with its all-reduce fused in. Returns (this rank's
        fp32 sum view [rows, hidden], sync tuple for the consuming RMSNorm)."""
        mode = ops.W4A16 if xq is None else ops.W4A8
        a = x if xq is None else xq
        rows = a.shape[0]
        n, k = linear.out_features, linear.in_features
        if split is None:
            split = linear.split(rows, True) if mode == ops.W4A16 else 1
        per = self.max_rows * self.hidden
        view = self.data[slot * per: slot * per + rows * n].view(rows, n)
        ops.wq_gemm_allreduce(mode, linear.qweight, linear.scales, a, view, self.data_mc + slot * per * 4,
                              self.flag_mc + slot * 8, xscale=xs, split=split, gemv_local=self.gemv_local[slot],
                              gemv_ticket=self.gemv_ticket[slot])
        expected = self.world * ops.wq_gemm_ctas(mode, rows, n, k, split)
        self.calls += 1
        return view, (self.flags[slot:slot + 1], self.state[slot], expected)
