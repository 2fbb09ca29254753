"""Sequence parallelism for tensor-parallel prefill, with the collectives fused
into the GEMMs.

Under TP the row-parallel projections (o_proj, down_proj) end in an all-reduce
of their ``[T, hidden]`` output (the reference runs vLLM's oneCCL all-reduce
there, ``k8v4_v030/launch.sh:101-110``; it cost 8.7 s of a 64K prefill on its
two GPUs, ``docs/historical-benchmarks.md:39-44``). Here a prefill chunk
instead keeps the residual stream sharded by token rows between them:

* rank ``o`` owns the chunk's 128-row token tiles ``tile0[o] .. tile0[o + 1]``
  (contiguous, as even as whole tiles allow);
* GEMM -> reduce-scatter: each CTA of o_proj / down_proj stores its bf16
  partial rows straight into the owner's slot for this rank (peer memory over
  NVLink) and adds 1 to the owner's counter (``ops.wq_gemm_sp`` with
  ``rs_dst``), so early tiles travel while later ones compute;
* the owner's norm (``ops.rmsnorm_sp``) waits for every rank's CTAs, sums the
  slots in fp32 with the residual, normalizes, and pushes the normed rows
  (bf16, or int8 + scale for the W4A8 MLP) to every rank at once through the
  NVLS multicast address of a symmetric buffer, one signal per row;
* all-gather -> GEMM: the qkv / gate-up GEMM (``ops.wq_gemm_sp`` with
  ``ag_flag``) reads the gathered rows from this rank's copy; its CTAs start at
  this rank's own tiles and each waits (bounded) for its tile's owner.

Every counter only grows; the host tracks the cumulative number of signals
each wait needs (every rank computes the same numbers from the chunk sizes),
so nothing is reset between calls. Each wait is bounded and reports a timeout
through the status word.

Buffers are reused call after call without extra barriers, because every
rewrite sits behind a wait that needs the reading ranks' later work:
* rank A's next GEMM into rank B's slot s runs after A's all-gather GEMM that
  waited for B's rows of the next norm, which B only pushes after its norm
  that read slot s (stream order; every kernel waits for its predecessor);
* rank B's next push into a gathered buffer follows B's norm wait for every
  rank's reduce-scatter signals, which each rank sends only after its GEMM
  that read that buffer.
"""
from __future__ import annotations

import os

import torch
import torch.distributed as dist

from .. import ops

TILE = 128
SLOTS = 2      # o_proj -> slot 0, down_proj -> slot 1
GATHERS = 3    # 0: bf16 rows for qkv, 1: int8 rows (+ scales) for a W4A8 gate/up, 2: bf16 rows for a W4A16 gate/up


def sp_mode() -> str:
    """``K8V4_TP_PREFILL`` = ``nccl`` (default: each row-parallel GEMM
    followed by an NCCL all-reduce; measured 6 % faster at TP2) or ``sp``
    (the fused reduce-scatter / all-gather prefill where the box supports
    multicast)."""
    mode = os.environ.get("K8V4_TP_PREFILL", "nccl").strip().lower()
    if mode not in ("sp", "nccl"):
        raise ValueError("K8V4_TP_PREFILL must be sp or nccl, got %r" % mode)
    return mode


def tile_owners(rows: int, world: int) -> list[int]:
    """``tile0``: rank o owns token tiles [tile0[o], tile0[o + 1]) of a chunk of
    ``rows`` rows (contiguous runs, sizes differing by at most one tile)."""
    if rows < 1 or world < 1:
        raise ValueError("rows and world must be positive")
    tiles = -(-rows // TILE)
    return [o * tiles // world for o in range(world + 1)]


def owned_rows(rows: int, tile0: list[int], rank: int) -> tuple[int, int]:
    """(first row, row count) of rank ``rank``'s part of the chunk."""
    r0 = min(rows, tile0[rank] * TILE)
    r1 = min(rows, tile0[rank + 1] * TILE)
    return r0, r1 - r0


class SeqParallel:
    """Buffers, ownership and signal bookkeeping of one TP group's fused
    reduce-scatter / all-gather prefill."""

    def __init__(self, group, device: torch.device, max_rows: int, hidden: int):
        import torch.distributed._symmetric_memory as symm_mem
        self.group = group if group is not None else dist.group.WORLD
        self.world = dist.get_world_size(self.group)
        self.rank = dist.get_rank(self.group)
        if not 2 <= self.world <= 8:
            raise ValueError("sequence parallelism runs on 2 to 8 ranks")
        self.device = torch.device(device)
        self.max_rows = int(max_rows)
        self.hidden = int(hidden)
        tiles = -(-self.max_rows // TILE)
        self.max_local = -(-tiles // self.world) * TILE       # rows one rank can own
        self.padded = tiles * TILE                            # gathered rows
        H, W = self.hidden, self.world
        self.slot_elems = self.max_local * H                  # one source's slot
        mk = symm_mem.empty
        self.slots = mk(SLOTS * W * self.slot_elems, dtype=torch.bfloat16, device=self.device)
        self.gbf = mk(2 * self.padded * H, dtype=torch.bfloat16, device=self.device)     # gathers 0 and 2
        self.gq = mk(self.padded * H, dtype=torch.int8, device=self.device)              # gather 1 codes
        self.gs = mk(self.padded, dtype=torch.float32, device=self.device)               # gather 1 scales
        self.cnt = mk(64, dtype=torch.int64, device=self.device)
        for t in (self.slots, self.gbf, self.gq, self.gs, self.cnt):
            t.zero_()
        name = self.group.group_name
        hs = symm_mem.rendezvous(self.slots, name)
        hb = symm_mem.rendezvous(self.gbf, name)
        hq = symm_mem.rendezvous(self.gq, name)
        hsc = symm_mem.rendezvous(self.gs, name)
        hc = symm_mem.rendezvous(self.cnt, name)
        self._handles = (hs, hb, hq, hsc, hc)
        for h in (hb, hq, hsc, hc):
            if not h.has_multicast_support or int(h.multicast_ptr) == 0:
                raise RuntimeError("symmetric memory on this box has no multicast (NVLS) support")
        self.slot_peer = [int(p) for p in hs.buffer_ptrs]     # every rank's slots, in this process
        self.cnt_peer = [int(p) for p in hc.buffer_ptrs]
        self.gbf_mc, self.gq_mc, self.gs_mc, self.cnt_mc = (int(h.multicast_ptr) for h in (hb, hq, hsc, hc))
        self.residual = torch.zeros((self.max_local, H), dtype=torch.bfloat16, device=self.device)
        # cumulative signal counts each wait needs
        self.rs_target = [0] * SLOTS                          # signals into this rank's slots
        self.ag_target = [[0] * W for _ in range(GATHERS)]    # rows received from each source
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)                        # every copy is zero before the first signal
        self.rows = 0
        self.tile0: list[int] = []
        self.calls = 0

    # ------------------------------------------------------------- layout
    def fits(self, rows: int, hidden: int) -> bool:
        """Chunks where every rank owns at least one 128-row tile (smaller
        steps take the NCCL all-reduce: their collectives are latency, not
        bandwidth, and a rank without rows would only wait)."""
        return TILE * self.world <= rows <= self.max_rows and hidden == self.hidden

    def begin(self, rows: int) -> None:
        """Set up a chunk of ``rows`` token rows."""
        if not self.fits(rows, self.hidden):
            raise ValueError("chunk of %d rows does not fit (max %d)" % (rows, self.max_rows))
        self.rows = rows
        self.tile0 = tile_owners(rows, self.world)
        self.row0, self.nrows = owned_rows(rows, self.tile0, self.rank)

    def _rows_of(self, o: int) -> int:
        return owned_rows(self.rows, self.tile0, o)[1]

    def _tiles_of(self, o: int) -> int:
        return self.tile0[o + 1] - self.tile0[o]

    def _cnt_index_rs(self, slot: int) -> int:
        return slot

    def _cnt_index_ag(self, gather: int, src: int) -> int:
        return 8 + gather * 8 + src

    def slot_view(self, slot: int) -> torch.Tensor:
        n = self.world * self.slot_elems
        return self.slots[slot * n:(slot + 1) * n]

    # ------------------------------------------------------------- norms
    def norm_push(self, w: torch.Tensor, eps: float, gather: int, slot: int | None = None,
                  x_local: torch.Tensor | None = None) -> None:
        """Residual add + RMSNorm of this rank's rows, pushed to every rank's
        gathered buffer ``gather`` (0 / 2: bf16; 1: int8 + scales). The input
        is reduce-scatter ``slot`` (its signals are waited for) or, for the
        first layer, ``x_local`` (this rank's rows; it starts the residual)."""
        H, W = self.hidden, self.world
        rs_flag = rs_target = 0
        slots = None
        if slot is not None:
            self.rs_target[slot] += W * (H // TILE) * self._tiles_of(self.rank)
            rs_flag = self.cnt.data_ptr() + 8 * self._cnt_index_rs(slot)
            rs_target = self.rs_target[slot]
            slots = self.slot_view(slot)
        elif x_local is None:
            raise ValueError("norm_push needs a slot or x_local")
        y = yq = ys = 0
        if gather == 1:
            yq, ys = self.gq_mc, self.gs_mc
        else:
            y = self.gbf_mc + (0 if gather == 0 else self.padded * H * 2)
        ops.rmsnorm_sp(self.residual, w, self.nrows, eps, slots=slots, world=W, slot_stride=self.slot_elems,
                       x_local=x_local, init_residual=slot is None, rs_flag=rs_flag, rs_target=rs_target,
                       y=y, yq=yq, ys=ys, row0=self.row0, mc=True,
                       ag_sig=self.cnt_mc + 8 * self._cnt_index_ag(gather, self.rank))
        for o in range(W):
            self.ag_target[gather][o] += self._rows_of(o)

    def final_norm(self, w: torch.Tensor, eps: float, slot: int) -> torch.Tensor:
        """The last layer's residual add + norm of this rank's rows (local bf16)."""
        H, W = self.hidden, self.world
        self.rs_target[slot] += W * (H // TILE) * self._tiles_of(self.rank)
        out = torch.empty((max(1, self.nrows), H), dtype=torch.bfloat16, device=self.device)
        ops.rmsnorm_sp(self.residual, w, self.nrows, eps, slots=self.slot_view(slot), world=W,
                       slot_stride=self.slot_elems, rs_flag=self.cnt.data_ptr() + 8 * self._cnt_index_rs(slot),
                       rs_target=self.rs_target[slot], y=out.data_ptr(), row0=0, mc=False)
        return out[: self.nrows]

    # ------------------------------------------------------------- GEMMs
    def gathered(self, gather: int):
        """This rank's copy of gathered buffer ``gather`` over the chunk:
        ``(x, xscale)``."""
        H, M = self.hidden, self.rows
        if gather == 1:
            return self.gq[: M * H].view(M, H), self.gs[:M]
        off = 0 if gather == 0 else self.padded * H
        return self.gbf[off: off + M * H].view(M, H), None

    def gemm_ag(self, linear, gather: int) -> torch.Tensor:
        """All-gather -> GEMM: ``linear`` over every row of the chunk."""
        x, xs = self.gathered(gather)
        mode = ops.W4A8 if gather == 1 else ops.W4A16
        flag = self.cnt.data_ptr() + 8 * self._cnt_index_ag(gather, 0)
        self.calls += 1
        return ops.wq_gemm_sp(mode, linear.qweight, linear.scales, x, self.world, self.rank, self.tile0,
                              xscale=xs, ag_flag=flag, ag_target=self.ag_target[gather])

    def gemm_rs(self, linear, slot: int, x: torch.Tensor | None = None, xq: torch.Tensor | None = None,
                xs: torch.Tensor | None = None) -> None:
        """GEMM -> reduce-scatter: ``linear``'s bf16 partial rows go into the
        owners' ``slot`` for this rank; the owners' norms sum them."""
        mode = ops.W4A16 if xq is None else ops.W4A8
        a = x if xq is None else xq
        per = self.world * self.slot_elems * 2            # bytes of one slot on each rank
        dst = [self.slot_peer[o] + slot * per + self.rank * self.slot_elems * 2 for o in range(self.world)]
        sig = [self.cnt_peer[o] + 8 * self._cnt_index_rs(slot) for o in range(self.world)]
        self.calls += 1
        ops.wq_gemm_sp(mode, linear.qweight, linear.scales, a, self.world, self.rank, self.tile0, xscale=xs,
                       rs_dst=dst, rs_sig=sig)

    def gather_rows(self, local: torch.Tensor, rows: torch.Tensor, comm) -> torch.Tensor:
        """Rows ``rows`` (global chunk indices) of the row-sharded ``local``
        ([nrows, H]) on every rank: each rank fills the ones it owns, then a
        sum over the group."""
        out = torch.zeros((rows.numel(), self.hidden), dtype=local.dtype, device=self.device)
        mine = (rows >= self.row0) & (rows < self.row0 + self.nrows)
        idx = mine.nonzero().flatten()
        if idx.numel():
            out.index_copy_(0, idx, local.index_select(0, rows[idx] - self.row0))
        comm.all_reduce(out)
        return out
