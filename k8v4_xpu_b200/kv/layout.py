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
        if self.fmt.name == "ref":
            if self.hkv not in (2, 4) or self.gqa != GQA:
                raise ValueError(
                    "unsupported per-GPU KV head count %r (ref K8/V4 serves 2 or 4, GQA 6)"
                    % (self.hkv,)
                )
        else:
            if self.hkv not in (1, 2, 4):
                raise ValueError("unsupported per-GPU KV head count %r" % (self.hkv,))
            if self.gqa not in (3, 6):
                raise ValueError("unsupported per-rank GQA %r" % (self.gqa,))

    @classmethod
    def for_heads(cls, num_heads: int, num_kv_heads: int, fmt: KVFormat | str = REF_FORMAT) -> "PageLayout":
        """Layout for one rank's local heads; a mismatched pair fails loudly."""
        if isinstance(fmt, str):
            fmt = FORMATS[fmt]
        num_heads = int(num_heads)
        num_kv_heads = int(num_kv_heads)
        if num_kv_heads < 1 or num_heads % num_kv_heads:
            raise ValueError("%d Q heads do not group over %d KV heads" % (num_heads, num_kv_heads))
        gqa = num_heads // num_kv_heads
        if fmt.name == "ref" and (num_kv_heads not in (2, 4) or gqa != GQA):
            raise ValueError(
                "K8/V4 serves 12/2 (TP2) or 24/4 (single GPU) local heads, got %d Q / %d KV"
                % (num_heads, num_kv_heads)
            )
        return cls(num_kv_heads, gqa, fmt)

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


def expand_block_ids(block_ids: list[int], ratio: int) -> list[int]:
    """Manager block id -> kernel pages (``block_id * ratio + sub``)."""
    ratio = int(ratio)
    if ratio < 1:
        raise ValueError("pages_per_block must be >= 1")
    out: list[int] = []
    for block_id in block_ids:
        base = int(block_id) * ratio
        out.extend(base + sub for sub in range(ratio))
    return out


def visible_lens(seq_len: int, q_len: int, max_t: int = DECODE_MAX_T) -> list[int]:
    """Per-query causal ends for one MTP step.

    Index 0 is the longest end (the page-valid length); index ``1+j`` is the
    end for query ``j``: ``seq_len - (q_len - 1 - j)``, clamped at 1. Lengths
    are full integers; a length near 59.5K must not be narrowed to 16 bits.
    Behaviour of ``k8v4_v030/layout.py:124-139``.
    """
    q_len = int(q_len)
    seq_len = int(seq_len)
    if q_len < 1 or q_len > max_t:
        raise ValueError("q_len %d outside packed decode tile" % q_len)
    rows = []
    for j in range(q_len):
        end = seq_len - (q_len - 1 - j)
        rows.append(end if end >= 1 else 1)
    return [max(rows)] + rows


def builtin_q_end(seq_len: int, q_len: int, q_tok: int) -> int:
    """Causal end of query ``q_tok`` of the last ``q_len`` tokens."""
    return int(seq_len) - int(q_len) + int(q_tok) + 1


def as_int16(value: int) -> int:
    """The reference's historic ABI bug: a length narrowed to signed 16 bits."""
    masked = int(value) & 0xFFFF
    return masked - 0x10000 if masked >= 0x8000 else masked


# -------------------------------------------------------------------- regions
def page_regions(page_index: int, layout: PageLayout, head: int | None = None) -> dict[str, tuple[int, int]]:
    """Byte offset and length of each region of one page.

    Token-major pages have one region per kind for all heads. Head-major pages
    have one run per head; pass ``head`` to get that head's regions (without it
    the first head's run is described together with the page extent).
    """
    base = int(page_index) * layout.page_bytes
    fmt = layout.fmt
    if fmt.order == "token_major":
        k0 = base
        v0 = k0 + layout.k_bytes_per_page
        s0 = v0 + layout.v_bytes_per_page
        out = {
            "k": (k0, layout.k_bytes_per_page),
            "v": (v0, layout.v_bytes_per_page),
            "k_scale": (s0, layout.scale_bytes_per_page),
            "v_scale": (s0 + layout.scale_bytes_per_page, layout.v_scale_bytes_per_page),
        }
        if fmt.has_v_zero:
            out["v_zero"] = (s0 + layout.scale_bytes_per_page + layout.v_scale_bytes_per_page,
                             layout.scale_bytes_per_page)
        return out
    h = 0 if head is None else int(head)
    if h < 0 or h >= layout.hkv:
        raise IndexError(h)
    hb = base + h * layout.head_page_bytes
    kb = layout.page * fmt.head_dim
    vb = layout.page * fmt.v_cols
    sb = layout.page * fmt.scale_bytes
    out = {
        "k": (hb, kb),
        "v": (hb + kb, vb),
        "k_scale": (hb + kb + vb, sb),
        "v_scale": (hb + kb + vb + sb, sb * fmt.v_groups),
    }
    if fmt.has_v_zero:
        out["v_zero"] = (hb + kb + vb + sb * (1 + fmt.v_groups), sb)
    return out


def block_byte_span(block_id: int, block_size: int, layout: PageLayout) -> tuple[int, int]:
    """Start and length of one manager block in the packed blob."""
    ratio = pages_per_block(block_size, layout.page)
    start = int(block_id) * ratio * layout.page_bytes
    return start, ratio * layout.page_bytes


def attention_pages_per_block(manager_block: int, kernel_block: int | None, page: int = PAGE) -> int:
    """How many kernel pages one block-table entry stands for.

    A ``page``-token kernel block is one page; a larger entry expands as
    ``block_id * ratio + page_in_block`` (the page ``slot // page`` writes).
    ``kernel_block is None`` means the table is still in manager blocks.
    """
    manager_block = int(manager_block)
    if manager_block < page or manager_block % page != 0:
        raise ValueError("manager block %s is not a multiple of %s" % (manager_block, page))
    if kernel_block is None:
        return manager_block // page
    kernel_block = int(kernel_block)
    if kernel_block == page:
        return 1
    if kernel_block < page or kernel_block % page != 0:
        raise ValueError("kernel block %s is not a multiple of %s" % (kernel_block, page))
    return kernel_block // page


def table_block_size(manager_block: int, kernel_block: int | None) -> int:
    """Token width of one block-table entry."""
    if kernel_block is None:
        return int(manager_block)
    return int(kernel_block)


def max_kernel_pages(max_model_len: int, manager_block: int, kernel_block: int | None, page: int = PAGE) -> int:
    """Kernel pages addressable by a full-length block table."""
    unit = table_block_size(manager_block, kernel_block)
    ratio = attention_pages_per_block(manager_block, kernel_block, page)
    width = (int(max_model_len) + unit - 1) // unit
    if width < 1:
        width = 1
    return width * ratio


def region_view_specs(num_pages: int, layout: PageLayout) -> dict[str, dict[str, object]]:
    """``as_strided`` specs for one contiguous run of pages.

    Strides are in elements of that region's dtype; ``byte_offset`` is from the
    start of page 0. Shapes are ``(pages, page, hkv, cols)`` for K/V/v_scale
    with more than one group and ``(pages, page, hkv)`` for per-row scales,
    whichever the page order, so callers index ``[page, token, head]``.
    """
    num_pages = int(num_pages)
    if num_pages < 1:
        raise ValueError("num_pages")
    fmt = layout.fmt
    sdt = fmt.scale_dtype
    sb = fmt.scale_bytes
    P, T, H, Dh, Vc, G = num_pages, layout.page, layout.hkv, fmt.head_dim, fmt.v_cols, fmt.v_groups
    pb = layout.page_bytes
    if pb % sb:
        raise ValueError("page bytes not a multiple of the scale size")
    specs: dict[str, dict[str, object]] = {}
    if fmt.order == "token_major":
        s0 = layout.k_bytes_per_page + layout.v_bytes_per_page
        specs["k"] = {"dtype": "int8", "shape": (P, T, H, Dh), "stride": (pb, H * Dh, Dh, 1), "byte_offset": 0}
        specs["v"] = {"dtype": "uint8", "shape": (P, T, H, Vc), "stride": (pb, H * Vc, Vc, 1),
                      "byte_offset": layout.k_bytes_per_page}
        specs["k_scale"] = {"dtype": sdt, "shape": (P, T, H), "stride": (pb // sb, H, 1), "byte_offset": s0}
        if G == 1:
            specs["v_scale"] = {"dtype": sdt, "shape": (P, T, H), "stride": (pb // sb, H, 1),
                                "byte_offset": s0 + layout.scale_bytes_per_page}
        else:
            specs["v_scale"] = {"dtype": sdt, "shape": (P, T, H, G), "stride": (pb // sb, H * G, G, 1),
                                "byte_offset": s0 + layout.scale_bytes_per_page}
        if fmt.has_v_zero:
            specs["v_zero"] = {"dtype": sdt, "shape": (P, T, H), "stride": (pb // sb, H, 1),
                               "byte_offset": s0 + layout.scale_bytes_per_page + layout.v_scale_bytes_per_page}
        return specs
    hp = layout.head_page_bytes
    kb, vb, ssb = T * Dh, T * Vc, T * sb
    specs["k"] = {"dtype": "int8", "shape": (P, T, H, Dh), "stride": (pb, Dh, hp, 1), "byte_offset": 0}
    specs["v"] = {"dtype": "uint8", "shape": (P, T, H, Vc), "stride": (pb, Vc, hp, 1), "byte_offset": kb}
    specs["k_scale"] = {"dtype": sdt, "shape": (P, T, H), "stride": (pb // sb, 1, hp // sb),
                        "byte_offset": kb + vb}
    if G == 1:
        specs["v_scale"] = {"dtype": sdt, "shape": (P, T, H), "stride": (pb // sb, 1, hp // sb),
                            "byte_offset": kb + vb + ssb}
    else:
        specs["v_scale"] = {"dtype": sdt, "shape": (P, T, H, G), "stride": (pb // sb, G, hp // sb, 1),
                            "byte_offset": kb + vb + ssb}
    if fmt.has_v_zero:
        specs["v_zero"] = {"dtype": sdt, "shape": (P, T, H), "stride": (pb // sb, 1, hp // sb),
                           "byte_offset": kb + vb + ssb * (1 + G)}
    return specs


_ELEM = {"int8": 1, "uint8": 1, "float32": 4, "float16": 2}


def element_byte(spec: dict[str, object], index: tuple[int, ...]) -> int:
    """Byte address of one element of a region spec."""
    shape = spec["shape"]
    stride = spec["stride"]
    if len(index) != len(shape) or len(stride) != len(shape):
        raise ValueError("index rank")
    elem = _ELEM[str(spec["dtype"])]
    off = int(spec["byte_offset"])
    for i, size, step in zip(index, shape, stride):
        i = int(i)
        if i < 0 or i >= int(size):
            raise IndexError(i)
        off += i * int(step) * elem
    return off


def region_stays_inside_block(block_size: int, layout: PageLayout) -> bool:
    """K, V and scales of every page sit inside that manager block."""
    ratio = pages_per_block(block_size, layout.page)
    start, length = block_byte_span(0, block_size, layout)
    end = start + length
    heads = range(layout.hkv) if layout.fmt.order == "head_major" else (None,)
    for page in range(ratio):
        for head in heads:
            for off, nbytes in page_regions(page, layout, head).values():
                if off < start or off + nbytes > end:
                    return False
    return True
