"""Gather-dequant kernel, backend end to end, eager oracle vs the CUDA kernels (GPU)."""
import pytest
import torch

from k8v4_xpu_b200 import ops
from k8v4_xpu_b200.attention.backend import K8V4AttentionImpl, K8V4MetadataBuilder
from k8v4_xpu_b200.attention.reference import eager_prefill
from k8v4_xpu_b200.kv.layout import b200_layout
from k8v4_xpu_b200.kv.pack import gather_sequence, store_tokens

pytestmark = pytest.mark.gpu


def _case(n, hkv=4, gqa=6, seed=0):
    g = torch.Generator().manual_seed(seed)
    lay = b200_layout(hkv, gqa)
    npg = (n + 15) // 16
    pages = torch.randperm(npg + 5, generator=g)[:npg]
    cache = torch.zeros(npg + 5, lay.page_bytes, dtype=torch.uint8)
    k = torch.randn(n, hkv, 128, generator=g).bfloat16()
    v = torch.randn(n, hkv, 128, generator=g).bfloat16()
    slots = (pages.repeat_interleave(16) * 16 + torch.arange(16).repeat(npg))[:n]
    store_tokens(cache, slots, k, v, lay)
    return lay, cache, pages


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_gather_dequant_bitwise_vs_torch(dtype):
    n = 1000
    lay, cache, pages = _case(n)
    kd, vd = gather_sequence(cache, pages.tolist(), n, lay)
    cd = cache.cuda()
    for h in range(lay.hkv):
        k, v = ops.gather_dequant(cd, pages.cuda(), lay.hkv, h, n, dtype=dtype)
        torch.cuda.synchronize()
        assert torch.equal(k.cpu(), kd[:, h].to(dtype))
        assert torch.equal(v.cpu(), vd[:, h].to(dtype))
    assert ops.status() == 0


def test_backend_decode_and_prefill_match_eager_oracle():
    hkv, gqa = 4, 6
    impl = K8V4AttentionImpl(hkv * gqa, 128, None, hkv)
    bld = K8V4MetadataBuilder(hkv * gqa, hkv, device="cuda")
    lay = b200_layout(hkv, gqa)
    g = torch.Generator().manual_seed(5)
    lens = [300, 47]
    tables = [list(range(0, 19)), list(range(19, 22))]
    cache = torch.zeros(32, lay.page_bytes, dtype=torch.uint8, device="cuda")
    # prefill both prompts through the backend (K/V written by do_kv_cache_update)
    T = sum(lens)
    q = torch.randn(T, hkv * gqa, 128, generator=g).bfloat16().cuda()
    k = torch.randn(T, hkv, 128, generator=g).bfloat16().cuda()
    v = torch.randn(T, hkv, 128, generator=g).bfloat16().cuda()
    slots = [t[p // 16] * 16 + p % 16 for t, n in zip(tables, lens) for p in range(n)]
    md = bld.build(lens, lens, tables, slots)
    assert not md.is_decode
    out = impl.forward(q, k, v, cache, md)
    torch.cuda.synchronize()
    off = 0
    for t, n in zip(tables, lens):
        ref = eager_prefill(q[off:off + n].cpu(), cache.cpu(), t, n, hkv, gqa, quant_q=True)
        err = (out[off:off + n].float().cpu() - ref).abs().max().item()
        assert err < 3e-2, err
        off += n
    # one decode token each (uniform packed), K/V appended at the next slot
    qd = torch.randn(2, hkv * gqa, 128, generator=g).bfloat16().cuda()
    kd = torch.randn(2, hkv, 128, generator=g).bfloat16().cuda()
    vd = torch.randn(2, hkv, 128, generator=g).bfloat16().cuda()
    new = [n + 1 for n in lens]
    md = bld.build([1, 1], new, tables, [t[n // 16] * 16 + n % 16 for t, n in zip(tables, lens)])
    assert md.is_decode
    od = impl.forward(qd, kd, vd, cache, md)
    torch.cuda.synchronize()
    for i, (t, n) in enumerate(zip(tables, new)):
        ref = eager_prefill(qd[i:i + 1].cpu(), cache.cpu(), t, n, hkv, gqa, quant_q=True)
        assert (od[i:i + 1].float().cpu() - ref).abs().max().item() < 3e-2
    assert ops.status() == 0


def test_prefill_refused_inside_graph_capture():
    impl = K8V4AttentionImpl(24, 128, None, 4)
    bld = K8V4MetadataBuilder(24, 4, device="cuda")
    lay = b200_layout(4, 6)
    cache = torch.zeros(4, lay.page_bytes, dtype=torch.uint8, device="cuda")
    md = bld.build([20], [20], [[0, 1]], list(range(20)))
    q = torch.randn(20, 24, 128, device="cuda").bfloat16()
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    with pytest.raises(RuntimeError, match="CUDA graph"):
        with torch.cuda.graph(g, stream=s):
            impl.forward(q, None, None, cache, md)
