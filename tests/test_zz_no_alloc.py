"""The allocation-free decode attention entry point, called through its C symbol.

``k8v4_decode_attn_noalloc`` serves callers that cannot allocate device
memory when they run attention (threads that must not call cudaMalloc,
embedders whose memory belongs to another allocator, hosts that forbid
allocations after start-up): its split-K scratch is a fixed array inside the
library (declared in ``csrc/k8v4_c_api.h``). This test calls it through its
exported C symbol with ctypes, exactly as such a caller would, and checks two
consecutive calls: bit for bit against the allocating entry point (the same
kernels on the same data), and against the fp32 torch attention reference of
the dequantized cache within the tolerance of the other decode tests.

The file name sorts last so that a run stopping at the first failure has run
every other test before this one.
"""
import ctypes
import math

import pytest
import torch

from k8v4_xpu_b200 import ops
from k8v4_xpu_b200.kv.layout import b200_layout
from k8v4_xpu_b200.kv.oracle import attention_ref
from k8v4_xpu_b200.kv.pack import gather_sequence, store_tokens

pytestmark = pytest.mark.gpu


def _lib():
    ops.require()
    lib = ctypes.CDLL(ops.extension_path())
    fn = lib.k8v4_decode_attn_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                   ctypes.c_int, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                   ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_float,
                   ctypes.c_void_p, ctypes.c_void_p]
    lib.k8v4_decode_attn_noalloc_max_floats.restype = ctypes.c_int64
    return lib


def _case(seed, hkv=4, gqa=6, lens=(700, 1500, 33), q_len=1):
    """Device inputs ``(q, cu, lens, bt, cache, hkv, gqa, q_len)`` of a paged
    decode step and the fp32 reference output on the CPU."""
    g = torch.Generator().manual_seed(seed)
    layout = b200_layout(hkv, gqa)
    pages = [(n + 15) // 16 for n in lens]
    total = sum(pages) + 2
    perm = torch.randperm(total, generator=g)
    cache = torch.zeros(total, layout.page_bytes, dtype=torch.uint8)
    bt = torch.zeros(len(lens), max(pages), dtype=torch.int32)
    off = 0
    for i, (n, npg) in enumerate(zip(lens, pages)):
        pg = perm[off:off + npg]
        off += npg
        bt[i, :npg] = pg.to(torch.int32)
        k = torch.randn(n, hkv, 128, generator=g).bfloat16()
        v = torch.randn(n, hkv, 128, generator=g).bfloat16()
        slots = (pg.repeat_interleave(16) * 16 + torch.arange(16).repeat(npg))[:n].to(torch.int64)
        store_tokens(cache, slots, k, v, layout)
    q = torch.randn(len(lens) * q_len, hkv * gqa, 128, generator=g).bfloat16()
    cu = torch.arange(0, len(lens) * q_len + 1, q_len, dtype=torch.int32)
    # fp32 reference of what the kernels compute: attention over the dequantized cache
    refs = []
    for i, n in enumerate(lens):
        kd, vd = gather_sequence(cache, bt[i, :pages[i]].tolist(), n, layout)
        ends = [n - q_len + 1 + t for t in range(q_len)]
        refs.append(attention_ref(q[i * q_len:(i + 1) * q_len].float(), kd, vd, ends, gqa))
    dev = "cuda"
    args = (q.to(dev), cu.to(dev), torch.tensor(lens, dtype=torch.int32, device=dev), bt.to(dev), cache.to(dev),
            hkv, gqa, q_len)
    return args, torch.cat(refs, 0)


def _call_noalloc(lib, q, cu, lens, bt, cache, hkv, gqa, q_len, nsplit, out):
    st = torch.cuda.current_stream().cuda_stream
    rc = lib.k8v4_decode_attn_noalloc(
        q.data_ptr(), cu.data_ptr(), lens.data_ptr(), None, bt.data_ptr(), bt.stride(0), cache.data_ptr(),
        cache.shape[0], hkv, 0, hkv, gqa, q.shape[1], lens.numel(), q_len, nsplit, 1.0 / math.sqrt(128),
        out.data_ptr(), st)
    return rc


@pytest.mark.parametrize("nsplit", [1, 5])
@pytest.mark.parametrize("q_len", [1, 7])
def test_noalloc_matches_allocating_entry_point_twice(q_len, nsplit):
    lib = _lib()
    for seed in (101, 202):  # two calls in a row on different data
        (q, cu, lens, bt, cache, hkv, gqa, ql), fp32_ref = _case(seed, q_len=q_len)
        ref = ops.decode_attn(q, cu, lens, bt, cache, hkv, gqa, ql, nsplit=nsplit)
        out = torch.full_like(q, float("nan"))
        rc = _call_noalloc(lib, q, cu, lens, bt, cache, hkv, gqa, ql, nsplit, out)
        torch.cuda.synchronize()
        assert rc == 0
        assert ops.status() == 0
        # the same kernels on the same data: equal bit for bit
        assert torch.equal(out, ref)
        err = (out.float().cpu() - fp32_ref).abs().max().item()
        assert err < 2e-2, err


def test_noalloc_rejects_oversized_launch():
    lib = _lib()
    (q, cu, lens, bt, cache, hkv, gqa, ql), _ = _case(7)
    cap = lib.k8v4_decode_attn_noalloc_max_floats()
    # pick a split count whose scratch exceeds the built-in array
    nsplit = 1
    while ops.decode_ws_floats(lens.numel(), hkv, nsplit, ql, gqa) <= cap:
        nsplit *= 2
    out = torch.zeros_like(q)
    rc = _call_noalloc(lib, q, cu, lens, bt, cache, hkv, gqa, ql, nsplit, out)
    assert rc == 20
