"""Page geometry, MTP causal ends and the int16 regression (CPU).

Behaviour of the reference's k8v4_v030/tests/test_layout_mtp.py, extended to
the parametric b200 format.
"""
import pytest

from k8v4_xpu_b200.kv import layout as L


REF2 = L.ref_layout(2)
REF4 = L.ref_layout(4)


def test_reference_format_bytes():
    assert L.GQA == 6 and L.SLOT_BYTES_PER_HEAD == 396
    for lay in (REF2, REF4):
        assert lay.hq == 6 * lay.hkv
        assert lay.bytes_per_token == 396 * lay.hkv
        assert lay.page_bytes == lay.bytes_per_token * L.PAGE
        assert lay.bytes_per_token < lay.fp8_bytes_per_token
    assert REF2.bytes_per_token == 792 and REF2.page_bytes == 50688 and REF2.fp8_bytes_per_token == 1024
    assert REF4.bytes_per_token == 1584 and REF4.page_bytes == 101376
    assert REF4.bytes_per_token > REF2.fp8_bytes_per_token
    assert L.CACHE_DTYPE == "int8_k_int4_v"


def test_reference_format_rejects_other_heads():
    for bad in (1, 3):
        with pytest.raises(ValueError):
            L.ref_layout(bad)
    with pytest.raises(ValueError):
        L.PageLayout.for_rank(12, 4)  # GQA 3 is not a reference deployment
    with pytest.raises(ValueError):
        L.PageLayout.for_rank(24, 2)  # GQA 12
    with pytest.raises(ValueError):
        L.PageLayout.for_rank(13, 2)  # heads do not group
    assert L.PageLayout.for_rank(12, 2).hkv == 2
    assert L.PageLayout.for_rank(12, 4, "b200").gqa == 3


def test_b200_format_geometry():
    fmt = L.B200_FORMAT
    assert fmt.slot_bytes_per_head == 128 + 64 + 2 + 8 == 202
    for hkv, gqa in ((4, 6), (2, 6), (1, 6), (1, 3)):
        lay = L.b200_layout(hkv, gqa)
        assert lay.page == 16 and lay.head_dim == 128
        assert lay.head_page_bytes == 3232 and lay.head_page_bytes % 16 == 0
        assert lay.page_bytes == hkv * 3232
        # every region of a head run starts 16-byte aligned (one bulk copy / TMA box each)
        for h in range(hkv):
            for off, n in L.page_regions(0, lay, h).values():
                assert off % 16 == 0 and n % 16 == 0
        assert lay.decode_max_t == 128 // gqa
        assert lay.bytes_per_token < lay.fp8_bytes_per_token
    assert L.b200_layout(4).bytes_per_token == 808
    with pytest.raises(ValueError):
        L.b200_layout(3)
    with pytest.raises(ValueError):
        L.b200_layout(1, 4)


@pytest.mark.parametrize("lay", [REF2, REF4, L.b200_layout(4), L.b200_layout(1, 3)])
def test_region_specs_address_every_byte_once(lay):
    pages = 3
    specs = L.region_view_specs(pages, lay)
    assert lay.regions_fill_page()
    seen = set()
    import itertools
    for name, spec in specs.items():
        elem = {"int8": 1, "uint8": 1, "float32": 4, "float16": 2}[spec["dtype"]]
        for idx in itertools.product(*[range(n) for n in spec["shape"]]):
            b = lay.byte_of(name, *idx)
            # the as_strided spec and the plane table address the same byte
            assert b == spec["byte_offset"] + elem * sum(i * s for i, s in zip(idx, spec["stride"]))
            for k in range(elem):
                assert b + k not in seen, (name, idx)
                seen.add(b + k)
    assert seen == set(range(pages * lay.page_bytes))
    with pytest.raises(IndexError):
        lay.byte_of("k", 0, lay.page, 0)
    with pytest.raises(IndexError):
        lay.byte_of("k", 0, 0, lay.hkv)


def test_slot_addressing_and_block_expansion():
    assert L.kernel_page_and_offset(-1) == (-1, -1)
    assert L.kernel_page_and_offset(130) == (2, 2)
    assert L.kernel_page_and_offset(130, 16) == (8, 2)
    assert L.expand_block_ids([3, 1], 2) == [6, 7, 2, 3]
    assert L.n_valid(100, 1) == 36 and L.n_valid(100, 2) == 0
    assert L.pages_per_block(2112) == 33
    with pytest.raises(ValueError):
        L.pages_per_block(100)
    assert L.attention_pages_per_block(2112, None) == 33
    assert L.attention_pages_per_block(2112, 64) == 1
    assert L.attention_pages_per_block(2112, 128) == 2
    assert L.max_kernel_pages(262144, 2112, None) == ((262144 + 2111) // 2112) * 33
    assert L.max_kernel_pages(262144, 2112, 128) == 262144 // 64
    geo = L.TableGeometry(2112, 128)
    assert geo.entry_tokens == 128 and geo.pages([5, 0]) == [10, 11, 0, 1]
    with pytest.raises(ValueError):
        L.TableGeometry(2112, 100)
    for lay in (REF2, L.b200_layout(2)):
        assert L.region_stays_inside_block(lay.page * 4, lay)


def test_visible_lens_and_int16_wrap():
    n = L.HISTORIC_MTP_LEN
    vis = L.visible_lens(n, 7)
    assert vis[0] == n and vis[1:] == [n - 6 + j for j in range(7)]
    assert all(v > 32767 for v in vis)
    assert L.as_int16(n) != n and L.as_int16(n) < 0  # the historic narrowing would corrupt it
    assert [L.as_int16(x) for x in (0, 32767, 32768, 65535, 65536, -1)] == [0, 32767, -32768, -1, 0, -1]
    assert L.visible_lens(3, 7)[1:5] == [1, 1, 1, 1]
    with pytest.raises(ValueError):
        L.visible_lens(100, 11)
    assert L.builtin_q_end(100, 7, 0) == 94 and L.builtin_q_end(100, 7, 6) == 100
    for seq in (59500, 59527, 63932, 70000):
        ends = [L.builtin_q_end(seq, 7, t) for t in range(7)]
        assert ends == L.visible_lens(seq, 7)[1:]
