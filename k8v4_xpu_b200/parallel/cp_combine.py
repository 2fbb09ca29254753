"""Context-parallel decode: the (m, l, O) partial exchange fused into the
decode attention kernel (peer stores over NVSwitch multicast).

Under context parallelism every rank's decode attention covers its own KV
pages; the split partials of all ranks are then merged into one output per
rank. The baseline exchange is an NCCL all-gather of each rank's workspace
between the attention kernel and the merge. Here instead:

* the decode kernel's epilogue stores each partial through the multicast
  address of this rank's slot in a symmetric gather buffer (``multimem.st``),
  so it lands in every rank's copy while the kernel's other CTAs still run;
* each CTA then adds 1 to a multicast counter (release, system scope);
* the merge kernel on every rank waits (bounded) until its copy of the counter
  holds every rank's CTAs, merges the slots from its own copy, and its last
  CTA advances a running count (so graph replays need no reset).

Two buffers alternate between calls. A rank writes buffer ``s`` again two
calls later, after its own merge of the call in between; that merge waited for
every rank's signals of that call, which each rank sends only after its merge
of the call that read buffer ``s``. So no rank still reads a slot that is
being overwritten.

``K8V4_CP_COMBINE`` = ``peer`` (default; the NCCL all-gather when the box has
no multicast) or ``nccl`` selects the exchange.
The reference has no context parallelism, so this module has no counterpart
there.
"""
from __future__ import annotations

import os

import torch
import torch.distributed as dist

from .. import ops

NUM_SMS = 148


def cp_combine_mode() -> str:
    mode = os.environ.get("K8V4_CP_COMBINE", "peer").strip().lower()
    if mode not in ("nccl", "peer"):
        raise ValueError("K8V4_CP_COMBINE must be nccl or peer, got %r" % mode)
    return mode


def max_slot_floats(max_seqs: int, hkv: int, max_q_len: int, gqa: int) -> int:
    """Floats of one rank's partials at the largest decode launch: at most one
    wave of CTAs (splits x sequences x heads <= the SM count), and at least two
    splits per (sequence, head)."""
    rows = max_q_len * gqa
    npad = 16 if rows <= 16 else 32 if rows <= 32 else 48 if rows <= 48 else 64
    ctas = max(NUM_SMS, 2 * max_seqs * hkv)
    return ctas * npad * (128 + 2)


def slot_layout(call: int, world: int, rank: int, rank_floats: int, slot_floats: int, slots: int = 2):
    """(buffer index, first float of the buffer, first float of this rank's
    slot) of exchange number ``call``: ranks' slots sit ``rank_floats`` apart
    inside buffer ``call % slots``, buffers ``world * slot_floats`` apart."""
    if rank_floats > slot_floats:
        raise ValueError("partials of %d floats exceed the slot of %d" % (rank_floats, slot_floats))
    b = call % slots
    base = b * world * slot_floats
    return b, base, base + rank * rank_floats


class PeerCombine:
    SLOTS = 2

    def __init__(self, group, device: torch.device, slot_floats: int):
        import torch.distributed._symmetric_memory as symm_mem
        self.group = group if group is not None else dist.group.WORLD
        self.world = dist.get_world_size(self.group)
        self.rank = dist.get_rank(self.group)
        self.device = torch.device(device)
        self.slot_floats = int(slot_floats)
        self.data = symm_mem.empty(self.SLOTS * self.world * self.slot_floats, dtype=torch.float32,
                                   device=self.device)
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
            raise RuntimeError("no multicast address for the partial exchange")
        if self.data_mc == self.data.data_ptr() or self.flag_mc == self.flags.data_ptr():
            # multimem instructions need a real multicast mapping, not the unicast buffer
            raise RuntimeError("the multicast address is the local buffer (no multicast object)")
        # per buffer: [signals consumed so far, merge CTAs done] (local to this rank)
        self.state = torch.zeros((self.SLOTS, 2), dtype=torch.int64, device=self.device)
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)  # every copy is initialised before the first store
        self.calls = 0

    def fits(self, rank_floats: int) -> bool:
        return rank_floats <= self.slot_floats

    def attention(self, q, cu_q, local_lens, local_bt, cache, hkv: int, gqa: int, max_q_len: int,
                  nsplit: int, q_ends=None) -> torch.Tensor:
        """This rank's decode attention over its own pages, exchanged and
        merged with every rank's: returns the full attention output.
        ``q_ends`` [T]: per-row visible local key counts (MTP verify rows)."""
        B = cu_q.numel() - 1
        rank_floats = ops.decode_ws_floats(B, hkv, nsplit, max_q_len, gqa)
        b, base, mine = slot_layout(self.calls, self.world, self.rank, rank_floats, self.slot_floats, self.SLOTS)
        ops.decode_attn_push(q, cu_q, local_lens, local_bt, cache, hkv, gqa, max_q_len, nsplit,
                             self.data_mc + 4 * mine, self.flag_mc + 8 * b, q_ends=q_ends)
        out = torch.empty_like(q)
        expected = self.world * ops.decode_push_ctas(B, hkv, nsplit)
        ops.decode_combine_ranks(self.data[base: base + self.world * rank_floats], rank_floats, cu_q, self.world,
                                 nsplit, hkv, gqa, max_q_len, out,
                                 sync=(self.flags[b:b + 1], self.state[b], expected))
        self.calls += 1
        return out
