"""Byte pack/unpack, strided cache views and the quantization rules (CPU)."""
import struct

import pytest
import torch

from k8v4_xpu_b200.kv import layout as L
from k8v4_xpu_b200.kv import oracle as O
from k8v4_xpu_b200.kv.pack import gather_sequence, read_token, store_tokens, write_token
from k8v4_xpu_b200.kv.views import allocate_cache, bind_regions, byte_run, span_problem


@pytest.mark.parametrize("lay", [L.ref_layout(2), L.ref_layout(4), L.b200_layout(4), L.b200_layout(1, 3)])
def test_write_read_roundtrip_and_vectorized_store(lay):
    g = torch.Generator().manual_seed(0)
    D = lay.head_dim
    n = lay.page + 5  # a partial second page
    k = torch.randn(n, lay.hkv, D, generator=g).bfloat16()
    v = torch.randn(n, lay.hkv, D, generator=g).bfloat16()
    slots = torch.arange(n) + lay.page  # start on page 1
    blob = bytearray(4 * lay.page_bytes)
    for t in range(n):
        write_token(blob, int(slots[t]), k[t].float().tolist(), v[t].float().tolist(), lay)
    cache = torch.zeros(4, lay.page_bytes, dtype=torch.uint8)
    store_tokens(cache, slots, k, v, lay)
    assert bytes(blob) == cache.numpy().tobytes()
    kd, vd = gather_sequence(cache, [1, 2], n, lay)
    kr, vr = O.quant_dequant_kv(k, v, lay)
    assert torch.equal(kd, kr) and torch.equal(vd, vr)
    kk, vv = read_token(blob, int(slots[3]), lay)
    assert torch.allclose(torch.tensor(kk), kd[3]) and torch.allclose(torch.tensor(vv), vd[3])
    # quantization error bounds: K within half a step, V within half a step
    kq, ks = O.quant_k_t(k.float(), lay.fmt.scale_dtype)
    assert (kd - k.float()).abs().max() <= ks.float().max() * 0.5 + 1e-6


def test_negative_and_out_of_range_slots_are_skipped():
    lay = L.b200_layout(2)
    cache = torch.zeros(2, lay.page_bytes, dtype=torch.uint8)
    k = torch.ones(3, 2, 128).bfloat16()
    store_tokens(cache, torch.tensor([-1, 2 * 16 + 3, -5]), k, k, lay)
    assert cache.count_nonzero() == 0
    blob = bytearray(lay.page_bytes)
    write_token(blob, -1, k[0].float().tolist(), k[0].float().tolist(), lay)
    assert not any(blob)


def test_reference_affine_v_edge_cases():
    # a row that spans zero dequantizes within half a step
    row = [(i - 100) / 37.0 for i in range(256)]
    packed, scale, zero = O.quant_v(row)
    assert 0 <= zero <= 15
    deq = O.dequant_v(packed, scale, zero)
    assert max(abs(a - b) for a, b in zip(deq, row)) <= scale * 0.5 + 1e-6
    # a constant row takes the 1e-8 scale floor (stored as fp32)
    _, scale, zero = O.quant_v([0.5] * 256)
    assert abs(scale - 1e-8) < 1e-14 and zero == 0.0
    # one-signed rows: the zero point clamps to [0, 15] and the far end saturates,
    # exactly as the reference's affine rule does
    pos = [1.0 + i / 50 for i in range(256)]
    packed, scale, zero = O.quant_v(pos)
    assert zero == 0.0 and max(b >> 4 for b in packed) == 15
    neg = [-1.0 - i / 50 for i in range(256)]
    packed, scale, zero = O.quant_v(neg)
    assert zero == 15.0 and min(b & 0xF for b in packed) == 0
    q, s = O.quant_k([0.0] * 256)
    assert s == 0.0 and q == [0] * 256


def test_k_rounding_is_half_to_even_on_the_stored_scale():
    x = torch.tensor([[2.5, -2.5, 127.0, 0.5] + [0.0] * 124])
    q, s = O.quant_k_t(x, "float32")
    assert float(s) == 1.0
    assert q[0, :4].tolist() == [2, -2, 127, 0]


def test_sym_group_v_nibbles():
    x = torch.zeros(1, 128)
    x[0, :32] = torch.linspace(-7, 7, 32)
    nib, sc = O.quant_v_sym_t(x)
    assert sc.dtype == torch.float16 and sc.shape == (1, 4)
    assert nib.min() >= 1 and nib.max() <= 15
    assert (nib[0, 32:] == 8).all()  # zero groups store code 8
    packed = O.pack_nibbles(nib)
    assert packed.shape == (1, 64)
    assert torch.equal(O.unpack_nibbles(packed), nib)
    assert int(packed[0, 0]) & 0xF == int(nib[0, 0])  # low nibble = even dim


def test_views_refuse_bad_layouts():
    lay = L.ref_layout(2)
    cache = allocate_cache(3, lay)
    views = bind_regions(cache, lay)
    assert views["k"].shape == (3, 64, 2, 256) and views["k_scale"].dtype == torch.float32
    views["k_scale"][1, 5, 1] = 3.25
    off = lay.byte_of("k_scale", 1, 5, 1)
    assert struct.unpack("<f", cache.flatten()[off:off + 4].numpy().tobytes())[0] == 3.25
    # vLLM-style logical [block, head, token, cell] with memory order [block, token, head, cell]
    blocks = torch.zeros(2, 64, 2, 396, dtype=torch.uint8).permute(0, 2, 1, 3)
    assert bind_regions(blocks, lay)["k"].shape[0] == 2
    with pytest.raises(RuntimeError):
        bind_regions(torch.zeros(2, 4, 64, 396, dtype=torch.uint8), lay)  # 4 heads, layout serves 2
    with pytest.raises(RuntimeError):
        byte_run(torch.zeros(4, 8, dtype=torch.uint8)[:, ::2])  # gapped
    with pytest.raises(RuntimeError):
        byte_run(torch.zeros(1, 8, dtype=torch.uint8).expand(4, 8))  # overlapping (stride 0)
    with pytest.raises(RuntimeError):
        byte_run(torch.zeros(4, 8, dtype=torch.float32))  # not bytes
    with pytest.raises(RuntimeError):
        bind_regions(torch.zeros(lay.page_bytes + 16, dtype=torch.uint8), lay)  # not whole pages
    with pytest.raises(RuntimeError):
        byte_run(torch.zeros(16, dtype=torch.uint8).as_strided((4, 4), (2, 1)))  # rows overlap
    with pytest.raises(RuntimeError):
        byte_run(torch.zeros(64, dtype=torch.uint8)[1:])  # not 16-byte aligned
    assert span_problem(torch.zeros(2, 3, 16, dtype=torch.uint8).permute(2, 0, 1)) is None  # dense, any order
