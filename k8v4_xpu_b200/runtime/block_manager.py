"""Paged KV block manager with hash-chained prefix caching.

A *block* is ``block_size`` tokens (a multiple of the 16-token K8/V4 page);
block id ``b`` owns pages ``b * ratio + i`` (the reference's block-to-page
expansion, ``k8v4_v030/layout.py:175-193``). Full blocks are content
addressed by a hash chain over token ids (block i's key hashes block i-1's
key with its tokens), so a prompt that shares a prefix with an earlier one
reuses its pages: refcounts keep shared blocks alive, cached blocks with no
user sit in an LRU list and are evicted only when the free list runs dry.
A block is published to the cache only once all of its tokens have been
written, and only full blocks are ever shared, so in-place writes never touch
a shared page; ``fork`` copies on write for the partially filled tail.
"""
from __future__ import annotations

import collections
import dataclasses
import hashlib
import struct


class CapacityError(RuntimeError):
    """Raised when the KV pool cannot hold a request (the launcher's fit signal).

    ``fit_tokens`` (when known) is the longest context the pool can hold; the
    launcher retries at that length, and only after this error.
    """

    def __init__(self, msg: str, fit_tokens: int | None = None):
        super().__init__(msg)
        self.fit_tokens = fit_tokens


def chain_hash(parent: bytes | None, tokens) -> bytes:
    h = hashlib.blake2b(digest_size=16)
    h.update(parent or b"\0")
    h.update(struct.pack("<%di" % len(tokens), *[int(t) for t in tokens]))
    return h.digest()


@dataclasses.dataclass
class BlockInfo:
    ref: int = 0
    key: bytes | None = None  # content hash when published


class BlockManager:
    def __init__(self, num_blocks: int, block_size: int = 16, page: int = 16, enable_prefix_caching: bool = True):
        if block_size % page:
            raise ValueError("block_size must be a multiple of the %d-token page" % page)
        self.num_blocks = int(num_blocks)
        self.block_size = int(block_size)
        self.ratio = block_size // page
        self.enable_prefix_caching = enable_prefix_caching
        self.info = [BlockInfo() for _ in range(self.num_blocks)]
        self.free: collections.deque[int] = collections.deque(range(self.num_blocks))
        # per-sequence table version: bumped whenever entries already handed
        # out may change (new table, replaced block, truncation, free), so a
        # device copy of a table can be extended instead of rewritten
        self.version: dict[int, int] = {}
        self._clock = 0
        self.cached: dict[bytes, int] = {}
        self.evictable: collections.OrderedDict[int, None] = collections.OrderedDict()
        self.tables: dict[int, list[int]] = {}
        self.keys: dict[int, list[bytes]] = {}  # per-seq hash chain of its full blocks
        # counters (exported as metrics)
        self.prefix_queries = 0
        self.prefix_hits = 0

    # ------------------------------------------------------------- capacity
    @property
    def num_free(self) -> int:
        return len(self.free) + len(self.evictable)

    def usage(self) -> float:
        return 1.0 - self.num_free / max(1, self.num_blocks)

    def blocks_for(self, tokens: int) -> int:
        return (int(tokens) + self.block_size - 1) // self.block_size

    def can_allocate(self, extra_blocks: int) -> bool:
        return extra_blocks <= self.num_free

    def _take(self) -> int:
        if self.free:
            b = self.free.popleft()
        elif self.evictable:
            b, _ = self.evictable.popitem(last=False)
            key = self.info[b].key
            if key is not None and self.cached.get(key) == b:
                del self.cached[key]
            self.info[b].key = None
        else:
            raise CapacityError("KV cache out of blocks")
        self.info[b].ref = 1
        return b

    def _ref(self, b: int) -> None:
        if self.info[b].ref == 0:
            self.evictable.pop(b, None)
        self.info[b].ref += 1

    def _unref(self, b: int) -> None:
        inf = self.info[b]
        inf.ref -= 1
        if inf.ref < 0:
            raise RuntimeError("block %d refcount underflow" % b)
        if inf.ref == 0:
            if inf.key is not None and self.enable_prefix_caching:
                self.evictable[b] = None
            else:
                inf.key = None
                self.free.append(b)

    # ---------------------------------------------------------- sequences
    def match_prefix(self, tokens) -> tuple[list[int], list[bytes]]:
        """Cached blocks covering the longest full-block prefix of ``tokens``."""
        blocks, keys = [], []
        if not self.enable_prefix_caching:
            return blocks, keys
        parent = None
        bs = self.block_size
        # never match the whole prompt: the last token must be computed for logits
        n_full = (len(tokens) - 1) // bs
        for i in range(n_full):
            key = chain_hash(parent, tokens[i * bs:(i + 1) * bs])
            b = self.cached.get(key)
            if b is None:
                break
            blocks.append(b)
            keys.append(key)
            parent = key
        return blocks, keys

    def allocate(self, seq_id: int, tokens, prefix: bool = True) -> int:
        """Create the table of a new sequence; returns the number of cached tokens."""
        if seq_id in self.tables:
            raise RuntimeError("sequence %d already allocated" % seq_id)
        hit, keys = self.match_prefix(tokens) if prefix else ([], [])
        self.prefix_queries += len(tokens)
        need = self.blocks_for(len(tokens)) - len(hit)
        if need > self.num_free - sum(1 for b in hit if self.info[b].ref == 0):
            raise CapacityError("KV cache cannot hold %d tokens" % len(tokens))
        for b in hit:
            self._ref(b)
        self.tables[seq_id] = list(hit)
        self.keys[seq_id] = list(keys)
        self._bump(seq_id)
        cached = len(hit) * self.block_size
        self.prefix_hits += cached
        return cached

    def ensure(self, seq_id: int, total_tokens: int) -> None:
        """Grow the table so it covers ``total_tokens`` tokens."""
        table = self.tables[seq_id]
        need = self.blocks_for(total_tokens) - len(table)
        if need > self.num_free:
            raise CapacityError("KV cache out of blocks")
        for _ in range(need):
            table.append(self._take())

    def publish(self, seq_id: int, tokens, computed: int) -> None:
        """Publish the full blocks whose ``computed`` tokens are all written."""
        if not self.enable_prefix_caching:
            return
        table = self.tables[seq_id]
        keys = self.keys[seq_id]
        bs = self.block_size
        n_full = min(int(computed) // bs, len(table))
        while len(keys) < n_full:
            i = len(keys)
            key = chain_hash(keys[-1] if keys else None, tokens[i * bs:(i + 1) * bs])
            keys.append(key)
            b = table[i]
            other = self.cached.get(key)
            if other is None:
                self.cached[key] = b
                self.info[b].key = key
            elif other != b:
                # identical content computed twice: share the published block
                self._ref(other)
                table[i] = other
                self._unref(b)
                self._bump(seq_id)

    def truncate(self, seq_id: int, tokens: int) -> None:
        """Drop blocks past ``tokens`` (speculative rollback)."""
        table = self.tables[seq_id]
        keep = self.blocks_for(tokens)
        if len(table) > keep:
            self._bump(seq_id)
        while len(table) > keep:
            self._unref(table.pop())
        keys = self.keys[seq_id]
        while len(keys) > tokens // self.block_size:
            keys.pop()

    def fork(self, parent: int, child: int, tokens: int) -> list[tuple[int, int]]:
        """Share the parent's full blocks; copy its partial tail block.

        Returns the (src_block, dst_block) copies the caller must perform on
        the device before either sequence writes again.
        """
        ptable = self.tables[parent]
        n_full = int(tokens) // self.block_size
        if len(ptable) > n_full and self.num_free < 1:  # fail before any refcount moves
            raise CapacityError("KV cache out of blocks")
        table = []
        for b in ptable[:n_full]:
            self._ref(b)
            table.append(b)
        copies = []
        if len(ptable) > n_full:
            nb = self._take()
            copies.append((ptable[n_full], nb))
            table.append(nb)
        self.tables[child] = table
        self.keys[child] = list(self.keys[parent][:n_full])
        self._bump(child)
        return copies

    def free_seq(self, seq_id: int) -> None:
        for b in reversed(self.tables.pop(seq_id, [])):
            self._unref(b)
        self.keys.pop(seq_id, None)
        # versions come from one clock, so a sequence allocated again (after
        # a preemption) never repeats an old version: dropping the entry is safe
        self.version.pop(seq_id, None)

    def _bump(self, seq_id: int) -> None:
        self._clock += 1
        self.version[seq_id] = self._clock

    def page_table(self, seq_id: int) -> list[int]:
        """Kernel pages of the sequence (block ids expanded by the page ratio)."""
        return self.pages_from(seq_id, 0)

    def num_pages(self, seq_id: int) -> int:
        return len(self.tables[seq_id]) * self.ratio

    def pages_from(self, seq_id: int, start: int) -> list[int]:
        """Kernel pages of the sequence from page ``start`` on."""
        r = self.ratio
        table = self.tables[seq_id]
        if r == 1:
            return table[start:]
        return [b * r + i for b in table[start // r:] for i in range(r)][start % r:]

    def slot(self, seq_id: int, pos: int) -> int:
        table = self.tables[seq_id]
        b = table[pos // self.block_size]
        return b * self.block_size + pos % self.block_size

    def check_invariants(self) -> None:
        refs = collections.Counter()
        for t in self.tables.values():
            refs.update(t)
        for b, inf in enumerate(self.info):
            if inf.ref != refs.get(b, 0):
                raise AssertionError("block %d ref %d != uses %d" % (b, inf.ref, refs.get(b, 0)))
        free = set(self.free)
        ev = set(self.evictable)
        if free & ev:
            raise AssertionError("block both free and evictable")
        for b in free | ev:
            if self.info[b].ref:
                raise AssertionError("free block %d has refs" % b)
        if len(free) + len(ev) + sum(1 for i in self.info if i.ref) != self.num_blocks:
            raise AssertionError("blocks lost")
