"""Parametric K8/V4 page geometry.

A KV page holds ``page`` tokens of every local KV head: int8 K, packed int4 V
and the scales needed to dequantize both. Two formats are registered:

``ref``
    The reference deployment format (``k8v4_v030/layout.py:16-26,153-166``):
    head_dim 256, 64-token pages, token-major regions
    ``[K page*hkv*256][V page*hkv*128][k_scale f32][v_scale f32][v_zero f32]``,
    V affine per row. It is kept bit-exact so the reference behaviour tests
    (int16 wrap, partial pages, negative slots) port one to one.

``b200``
    The benchmark format: head_dim 128, 16-token pages, V symmetric int4 with
    one fp16 scale per 32-element group along head_dim, K symmetric int8 with
    an fp16 per-token-per-head scale. Pages are *head-major*: each (page, head)
    is one contiguous 3,232-byte run ``[K 16x128][V 16x64][k_scale 16][v_scale
    16x4]`` whose region offsets are all 16-byte aligned, so a single bulk copy
    (or one TMA box per region) moves a head's page into shared memory.

Nothing here reads the environment; byte-level code carries an explicit
:class:`PageLayout`.
"""
from __future__ import annotations

import dataclasses
import functools

CACHE_DTYPE = "int8_k_int4_v"
HISTORIC_MTP_LEN = 59500
# Rows of the attention kernels' query tile (one tcgen05 M=128 accumulator).
ATTN_TILE_ROWS = 128

_SCALE_BYTES = {"float32": 4, "float16": 2}


@dataclasses.dataclass(frozen=True)
class KVFormat:
    """Byte format of one K8/V4 page (independent of the head count)."""

    name: str
    head_dim: int
    page: int
    v_mode: str  # "affine_row" or "sym_group"
    v_group: int  # elements per V scale group; head_dim for affine_row
    scale_dtype: str  # "float32" or "float16"
    order: str  # "token_major" or "head_major"

    def __post_init__(self) -> None:
        if self.v_mode not in ("affine_row", "sym_group"):
            raise ValueError("v_mode %r" % (self.v_mode,))
        if self.scale_dtype not in _SCALE_BYTES:
            raise ValueError("scale_dtype %r" % (self.scale_dtype,))
        if self.order not in ("token_major", "head_major"):
            raise ValueError("order %r" % (self.order,))
        if self.head_dim % 32 or self.head_dim <= 0:
            raise ValueError("head_dim must be a positive multiple of 32")
        if self.head_dim % self.v_group:
            raise ValueError("v_group must divide head_dim")

    @property
    def scale_bytes(self) -> int:
        return _SCALE_BYTES[self.scale_dtype]

    @property
    def v_groups(self) -> int:
        """V scales per token per head (1 for affine rows)."""
        return self.head_dim // self.v_group

    @property
    def v_cols(self) -> int:
        """Packed V bytes per token per head (two int4 per byte)."""
        return self.head_dim // 2

    @property
    def has_v_zero(self) -> bool:
        return self.v_mode == "affine_row"

    @property
    def slot_bytes_per_head(self) -> int:
        """Bytes one token of one head occupies, scales included."""
        scales = 1 + self.v_groups + (1 if self.has_v_zero else 0)
        return self.head_dim + self.v_cols + scales * self.scale_bytes


REF_FORMAT = KVFormat("ref", 256, 64, "affine_row", 256, "float32", "token_major")
B200_FORMAT = KVFormat("b200", 128, 16, "sym_group", 32, "float16", "head_major")
FORMATS = {"ref": REF_FORMAT, "b200": B200_FORMAT}

# Reference-format constants, same values as the reference module constants.
PAGE = REF_FORMAT.page
D = REF_FORMAT.head_dim
GQA = 6
V4_COLS = D // 2
SLOT_BYTES_PER_HEAD = REF_FORMAT.slot_bytes_per_head  # 396
DECODE_MAX_T = PAGE // GQA  # 10


@dataclasses.dataclass(frozen=True)
class Region:
    """One typed plane of a page, with the byte steps that address it.

    Element ``(token, head, col)`` of page ``p`` sits at byte
    ``p * page_bytes + offset + token * token_step + head * head_step + col * elem``.
    ``cols`` is 1 for a per-(token, head) scalar such as ``k_scale``.
    """

    name: str
    dtype: str
    cols: int
    offset: int
    token_step: int
    head_step: int

    @property
    def elem(self) -> int:
        return _ELEM_BYTES[self.dtype]

    @property
    def row_bytes(self) -> int:
        """Bytes of one (token, head) entry."""
        return self.cols * self.elem


_ELEM_BYTES = {"int8": 1, "uint8": 1, "float32": 4, "float16": 2}


@dataclasses.dataclass(frozen=True)
class PageLayout:
    """Per-rank head layout plus the page format it is stored in.

    ``hkv`` is the number of KV heads this rank stores, ``gqa`` the number of
    query heads per KV head on this rank. The ``ref`` format only serves the
    reference's two deployments (2 or 4 KV heads, GQA 6); ``b200`` serves
    1, 2 or 4 KV heads with GQA 6 (TP1/2/4) or 3 (TP8, KV heads replicated).
    """

    hkv: int
    gqa: int = GQA
    fmt: KVFormat = REF_FORMAT

    def __post_init__(self) -> None:
        allowed = ({2, 4}, {GQA}) if self.fmt.name == "ref" else ({1, 2, 4}, {3, 6})
        if self.hkv not in allowed[0] or self.gqa not in allowed[1]:
            raise ValueError(
                "the %s page format stores %s KV heads per rank at GQA %s; asked for %r KV heads at GQA %r"
                % (self.fmt.name, sorted(allowed[0]), sorted(allowed[1]), self.hkv, self.gqa))

    @classmethod
    def for_rank(cls, hq_local: int, hkv_local: int, fmt: KVFormat | str = REF_FORMAT) -> "PageLayout":
        """Layout of a rank holding ``hq_local`` query and ``hkv_local`` KV
        heads; the constructor refuses a pair its format does not store."""
        fmt = FORMATS[fmt] if isinstance(fmt, str) else fmt
        groups, rest = divmod(int(hq_local), max(1, int(hkv_local)))
        if int(hkv_local) < 1 or rest:
            raise ValueError("%d query heads do not share %d KV heads evenly" % (hq_local, hkv_local))
        return cls(int(hkv_local), groups, fmt)

    # ------------------------------------------------------------------ sizes
    @property
    def page(self) -> int:
        return self.fmt.page

    @property
    def head_dim(self) -> int:
        return self.fmt.head_dim

    @property
    def hq(self) -> int:
        return self.gqa * self.hkv

    @property
    def decode_max_t(self) -> int:
        """Longest query one packed decode tile holds for one KV head."""
        if self.fmt.name == "ref":
            return self.page // self.gqa
        return ATTN_TILE_ROWS // self.gqa

    @property
    def k_bytes_per_page(self) -> int:
        return self.page * self.hkv * self.head_dim

    @property
    def v_bytes_per_page(self) -> int:
        return self.page * self.hkv * self.fmt.v_cols

    @property
    def scale_bytes_per_page(self) -> int:
        """Bytes of one per-token-per-head scale plane (k_scale)."""
        return self.page * self.hkv * self.fmt.scale_bytes

    @property
    def v_scale_bytes_per_page(self) -> int:
        return self.scale_bytes_per_page * self.fmt.v_groups

    @property
    def head_page_bytes(self) -> int:
        """Bytes of one (page, head) run in the head-major format."""
        return self.page * self.fmt.slot_bytes_per_head

    @property
    def page_bytes(self) -> int:
        return self.page * self.hkv * self.fmt.slot_bytes_per_head

    @property
    def bytes_per_token(self) -> int:
        return self.page_bytes // self.page

    @property
    def fp8_bytes_per_token(self) -> int:
        """fp8 K and V for the same local heads: 2 * head_dim bytes per head."""
        return self.hkv * 2 * self.head_dim

    @property
    def bf16_bytes_per_token(self) -> int:
        return self.hkv * 4 * self.head_dim

    # ---------------------------------------------------------------- regions
    @functools.cached_property
    def regions(self) -> tuple[Region, ...]:
        """The page's planes in storage order.

        The planes are K codes, V nibbles, K scales, V scales and (affine V
        only) V zero points. Token-major pages stack each plane for all heads
        (``[token][head][cols]``); head-major pages give every head one run
        holding all of its planes (``[head][plane][token][cols]``).
        """
        f = self.fmt
        sdt = f.scale_dtype
        planes = [("k", "int8", f.head_dim), ("v", "uint8", f.v_cols), ("k_scale", sdt, 1), ("v_scale", sdt, f.v_groups)]
        if f.has_v_zero:
            planes.append(("v_zero", sdt, 1))
        out, at = [], 0
        for name, dt, cols in planes:
            row = cols * _ELEM_BYTES[dt]
            if f.order == "token_major":
                out.append(Region(name, dt, cols, at, self.hkv * row, row))
                at += self.page * self.hkv * row
            else:  # offsets inside head 0's run; heads follow each other
                out.append(Region(name, dt, cols, at, row, self.head_page_bytes))
                at += self.page * row
        return tuple(out)

    def region(self, name: str) -> Region:
        for r in self.regions:
            if r.name == name:
                return r
        raise KeyError("no %r plane in the %s format" % (name, self.fmt.name))

    def byte_of(self, name: str, page: int, token: int, head: int, col: int = 0) -> int:
        """Address (from the start of page 0) of one element of a plane."""
        r = self.region(name)
        for what, i, n in (("token", token, self.page), ("head", head, self.hkv), ("col", col, r.cols)):
            if not 0 <= int(i) < n:
                raise IndexError("%s %d outside 0..%d" % (what, i, n - 1))
        if int(page) < 0:
            raise IndexError("page %d" % page)
        return int(page) * self.page_bytes + r.offset + int(token) * r.token_step + int(head) * r.head_step + int(col) * r.elem

    def extents(self, head: int | None = None) -> list[tuple[str, int, int]]:
        """``(plane, start, length)`` byte runs inside one page: one per plane
        for token-major pages, one per plane of ``head`` (every head when
        ``None``) for head-major pages."""
        if self.fmt.order == "token_major":
            return [(r.name, r.offset, self.page * self.hkv * r.row_bytes) for r in self.regions]
        heads = range(self.hkv) if head is None else [int(head)]
        return [(r.name, r.offset + h * r.head_step, self.page * r.row_bytes) for h in heads for r in self.regions]

    def regions_fill_page(self) -> bool:
        """The planes' runs cover ``[0, page_bytes)`` exactly once."""
        runs = sorted((start, length) for _n, start, length in self.extents())
        at = 0
        for start, length in runs:
            if start != at:
                return False
            at += length
        return at == self.page_bytes


def b200_layout(hkv: int, gqa: int = 6) -> PageLayout:
    return PageLayout(hkv, gqa, B200_FORMAT)


def ref_layout(hkv: int) -> PageLayout:
    return PageLayout(hkv, GQA, REF_FORMAT)


# ---------------------------------------------------------------------- slots
def pages_per_block(block_size: int, page: int = PAGE) -> int:
    block_size = int(block_size)
    if block_size < page or block_size % page != 0:
        raise ValueError("block_size must be a positive multiple of %d" % page)
    return block_size // page


def kernel_page_and_offset(slot: int, page: int = PAGE) -> tuple[int, int]:
    """Store addressing. Negative slots are skipped and never index a page."""
    slot = int(slot)
    if slot < 0:
        return -1, -1
    return slot // page, slot % page


def n_valid(seq_len: int, logical_page: int, page: int = PAGE) -> int:
    """Tokens of this page that belong to ``seq_len``; the tail is masked."""
    return max(0, min(page, int(seq_len) - int(logical_page) * page))


@dataclasses.dataclass(frozen=True)
class TableGeometry:
    """What one block-table entry stands for in kernel pages.

    The block manager hands out ``manager_block``-token blocks. A table given
    to the kernels is either still in those blocks (``kernel_block=None``) or
    re-expressed in ``kernel_block``-token entries; either way an entry covers
    ``entry_tokens`` tokens = ``pages_per_entry`` consecutive pages, and entry
    ``e`` names pages ``e * pages_per_entry ...`` (the pages ``slot // page``
    writes).
    """

    manager_block: int
    kernel_block: int | None = None
    page: int = PAGE

    def __post_init__(self) -> None:
        for what, n in (("manager block", self.manager_block), ("kernel block", self.kernel_block)):
            if n is not None and (int(n) < self.page or int(n) % self.page):
                raise ValueError("%s of %s tokens is not a whole number of %d-token pages" % (what, n, self.page))

    @property
    def entry_tokens(self) -> int:
        return int(self.manager_block if self.kernel_block is None else self.kernel_block)

    @property
    def pages_per_entry(self) -> int:
        return self.entry_tokens // self.page

    def pages(self, entries) -> list[int]:
        """Kernel pages of a list of table entries, in order."""
        n = self.pages_per_entry
        return [int(e) * n + i for e in entries for i in range(n)]

    def max_pages(self, max_model_len: int) -> int:
        """Pages a table wide enough for ``max_model_len`` tokens addresses."""
        entries = max(1, -(-int(max_model_len) // self.entry_tokens))
        return entries * self.pages_per_entry


def expand_block_ids(block_ids: list[int], ratio: int) -> list[int]:
    """Manager block id -> kernel pages (``block_id * ratio + sub``)."""
    if int(ratio) < 1:
        raise ValueError("a block spans at least one page, got %s" % ratio)
    return TableGeometry(int(ratio), None, 1).pages(block_ids)


def attention_pages_per_block(manager_block: int, kernel_block: int | None, page: int = PAGE) -> int:
    """How many kernel pages one block-table entry stands for."""
    return TableGeometry(manager_block, kernel_block, page).pages_per_entry


def max_kernel_pages(max_model_len: int, manager_block: int, kernel_block: int | None, page: int = PAGE) -> int:
    """Kernel pages addressable by a full-length block table."""
    return TableGeometry(manager_block, kernel_block, page).max_pages(max_model_len)


# ------------------------------------------------------- MTP causal query ends
def builtin_q_end(seq_len: int, q_len: int, q_tok: int) -> int:
    """Keys visible to query row ``q_tok`` of a ``q_len``-row step whose last
    row is token ``seq_len - 1``: its own position plus one."""
    return (int(seq_len) - int(q_len)) + int(q_tok) + 1


def visible_lens(seq_len: int, q_len: int, max_t: int = DECODE_MAX_T) -> list[int]:
    """The packed decode kernel's length vector for one MTP step.

    Entry 0 is the longest causal end (the page-valid length), then one end
    per query row, each at least 1. Lengths stay full integers: a length near
    59.5K must not be narrowed to 16 bits (``as_int16``).
    """
    if not 1 <= int(q_len) <= int(max_t):
        raise ValueError("a packed decode step holds 1..%d query rows, got %s" % (max_t, q_len))
    ends = [max(1, builtin_q_end(seq_len, q_len, r)) for r in range(int(q_len))]
    return [ends[-1]] + ends  # ends ascend, so the last row's is the longest


def as_int16(value: int) -> int:
    """``value`` as a two's-complement 16-bit integer: the historic ABI bug
    that narrowed sequence lengths (lengths above 32,767 turn negative)."""
    return ((int(value) + 0x8000) & 0xFFFF) - 0x8000


# -------------------------------------------------------------------- regions
def page_regions(page_index: int, layout: PageLayout, head: int | None = None) -> dict[str, tuple[int, int]]:
    """``{plane: (byte offset, length)}`` of one page (absolute offsets).

    Token-major pages have one run per plane for all heads; head-major pages
    one run per plane and head, so ``head`` picks the head (default 0).
    """
    base = int(page_index) * layout.page_bytes
    if layout.fmt.order == "head_major":
        h = 0 if head is None else int(head)
        if not 0 <= h < layout.hkv:
            raise IndexError(h)
        runs = layout.extents(h)
    else:
        runs = layout.extents()
    return {name: (base + start, length) for name, start, length in runs}


def region_stays_inside_block(block_size: int, layout: PageLayout) -> bool:
    """Every plane of every page of a ``block_size``-token manager block lies
    inside that block's bytes: the block holds whole pages and each page's
    planes tile the page."""
    whole = int(block_size) >= layout.page and int(block_size) % layout.page == 0
    return whole and layout.regions_fill_page()


def region_view_specs(num_pages: int, layout: PageLayout) -> dict[str, dict[str, object]]:
    """``as_strided`` arguments of each plane over ``num_pages`` pages.

    Shapes are ``(pages, page, hkv[, cols])`` (the column axis only when a
    plane holds more than one element per token and head), strides are in the
    plane's own elements, ``byte_offset`` counts from page 0.
    """
    if int(num_pages) < 1:
        raise ValueError("num_pages must be positive")
    specs: dict[str, dict[str, object]] = {}
    for r in layout.regions:
        e = r.elem
        if layout.page_bytes % e or r.token_step % e or r.head_step % e or r.offset % e:
            raise ValueError("plane %s is not aligned to its %d-byte elements" % (r.name, e))
        shape = (int(num_pages), layout.page, layout.hkv)
        stride = (layout.page_bytes // e, r.token_step // e, r.head_step // e)
        if r.cols > 1:
            shape, stride = shape + (r.cols,), stride + (1,)
        specs[r.name] = {"dtype": r.dtype, "shape": shape, "stride": stride, "byte_offset": r.offset}
    return specs
