"""Context parallelism (CP): the KV cache sharded by page across ranks.

The reference has no context parallelism; this is the long-context mechanism
of this framework (a KV-gather design, not ring attention):

* every CP rank holds the whole model (weights replicated) and a shard of
  every sequence's KV pages. A CP block is C pages, page j of block b on
  rank j at physical page b, so every rank's block manager (they all run the
  same one) agrees on where a page lives, and prefix caching works unchanged
  across the shard map;
* prefill: each rank runs the model on the chunk tokens whose pages it owns
  (so its KV writes stay local), then, in every layer, all ranks synchronize
  and the prefill attention kernel reads every page straight from its owner's
  cache (peer memory mapped into this process, per-source TMA maps; no
  multicast). The chunk's GEMMs are split C ways;
* decode: every rank runs the model on the new token (replicated GEMMs); the
  owner of the token's page writes its KV; each rank's decode attention
  covers its own pages and the (m, l, O) split partials of all ranks are
  exchanged and merged, so every rank continues with the same attention
  output. The exchange is an NCCL all-gather (``K8V4_CP_COMBINE=nccl``), or (the default)
  multicast stores from the attention kernel itself (``parallel.cp_combine``).

Every rank's KV pool lives in symmetric memory and is mapped into every
process (torch's symmetric-memory rendezvous does the handle exchange and
grants access); synchronization uses NCCL.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

PAGE = 16


def entry(src: int, page: int) -> int:
    """Block-table entry of a page on rank ``src``."""
    return (src << 24) | page


class CPGroup:
    def __init__(self, group=None):
        self.group = group if group is not None else dist.group.WORLD
        self.rank = dist.get_rank(self.group)
        self.world = dist.get_world_size(self.group)
        if self.world > 8:
            raise ValueError("context parallel size must be at most 8")
        self._peer_pools = None
        self._flag = None
        self.peer = None  # PeerCombine when the decode exchange runs through multicast stores

    # ----------------------------------------------------------- peer memory
    def alloc_pool(self, shape: tuple[int, ...], device) -> torch.Tensor:
        """This rank's KV pool in symmetric memory, with every rank's pool
        mapped into this process (torch's symmetric-memory rendezvous grants
        this GPU access to the peers' allocations)."""
        import torch.distributed._symmetric_memory as symm_mem
        pool = symm_mem.empty(*shape, dtype=torch.uint8, device=device)
        pool.zero_()
        h = symm_mem.rendezvous(pool, self.group.group_name)
        self._handle = h
        self._peer_pools = [pool if r == self.rank else h.get_buffer(r, tuple(shape), torch.uint8, 0)
                            for r in range(self.world)]
        torch.cuda.synchronize(device)
        dist.barrier(group=self.group)
        return pool

    def layer_caches(self, layer: int) -> list[torch.Tensor]:
        return [p[layer] for p in self._peer_pools]

    # ------------------------------------------------------------ collectives
    def sync(self, device) -> None:
        """Stream-ordered barrier: KV pages written before it are readable by every rank after it."""
        if self._flag is None or self._flag.device != torch.device(device):
            self._flag = torch.zeros(1, dtype=torch.float32, device=device)
        dist.all_reduce(self._flag, group=self.group)

    def all_gather(self, t: torch.Tensor) -> torch.Tensor:
        out = torch.empty((self.world * t.numel(),), dtype=t.dtype, device=t.device)
        dist.all_gather_into_tensor(out, t.reshape(-1).contiguous(), group=self.group)
        return out

    def sum_(self, t: torch.Tensor) -> torch.Tensor:
        dist.all_reduce(t, group=self.group)
        return t

    # ------------------------------------------------------------- page maps
    def owner(self, pos: int) -> int:
        return (pos // PAGE) % self.world

    def encoded_pages(self, blocks: list[int], n_tokens: int) -> list[int]:
        """Kernel block table of a sequence: logical page i -> (i % C, blocks[i // C])."""
        n_pages = (n_tokens + PAGE - 1) // PAGE
        C = self.world
        return [entry(i % C, blocks[i // C]) for i in range(n_pages)]

    def local_pages(self, blocks: list[int], n_tokens: int) -> tuple[list[int], int]:
        """This rank's pages of a sequence (physical ids, in order) and the keys they hold."""
        C, r = self.world, self.rank
        n_pages = (n_tokens + PAGE - 1) // PAGE
        pages, keys = [], 0
        for i in range(r, n_pages, C):
            pages.append(blocks[i // C])
            keys += min(PAGE, n_tokens - i * PAGE)
        return pages, keys

    def slot(self, blocks: list[int], pos: int) -> int:
        """Local slot of the token at ``pos`` on its owner, -1 on the other ranks."""
        if self.owner(pos) != self.rank:
            return -1
        return blocks[pos // (PAGE * self.world)] * PAGE + pos % PAGE

    def broadcast_(self, t: torch.Tensor) -> torch.Tensor:
        """Overwrite ``t`` with CP rank 0's copy, so that decisions the host
        takes from device results (accepted drafts, next tokens) are the same
        on every rank even where fp32 atomics left the ranks' sums a rounding
        apart."""
        dist.broadcast(t, src=dist.get_global_rank(self.group, 0), group=self.group)
        return t


def local_keys(n, rank: int, world: int):
    """Keys among a sequence's first ``n`` positions that CP rank ``rank``
    holds (its pages are logical pages rank, rank + world, ... of PAGE keys).

    Because a rank's pages are in position order, those keys are a prefix of
    its local key list: the keys that a query row at position ``n - 1`` may
    see. Works on ints and, elementwise, on integer tensors."""
    full = n // PAGE
    rem = n - full * PAGE
    # logical pages i < full with i % world == rank (never negative: rank < world)
    nfull = (full - rank + world - 1) // world
    if isinstance(n, torch.Tensor):
        return nfull * PAGE + torch.where(full % world == rank, rem, torch.zeros_like(rem))
    return nfull * PAGE + (rem if full % world == rank else 0)


def local_slots(blk: torch.Tensor, nblk: torch.Tensor, pos: torch.Tensor, rank: int, world: int) -> torch.Tensor:
    """Device form of :meth:`CPGroup.slot` for one position per sequence:
    ``blk`` [B, W] the sequences' block ids (zero padded), ``nblk`` [B] how
    many are real, ``pos`` [B] int64. -1 where another rank owns the page or
    the position lies past the sequence's blocks."""
    b = pos // (PAGE * world)
    own = ((pos // PAGE) % world == rank) & (b < nblk)
    page = blk.gather(1, b.clamp(max=blk.shape[1] - 1).view(-1, 1)).view(-1).to(torch.int64)
    return torch.where(own, page * PAGE + pos % PAGE, torch.full_like(pos, -1))
