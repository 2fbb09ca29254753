"""INT8 islands on the GPU: the W8A16 linear and a decoder forward with island layers."""
import pytest
import torch

from k8v4_xpu_b200 import ops
from k8v4_xpu_b200.layers.linear import Int8IslandLinear
from k8v4_xpu_b200.models import gptq
from k8v4_xpu_b200.models.config import TINY
from k8v4_xpu_b200.models.dense import DenseModel

from test_engine_gpu import _inputs

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("n", [384, 200])
def test_island_linear_matches_fp32_reference(n):
    """The in-tree int8 GEMM over two activation limbs (rows padded to the
    GEMM's tile for n = 200) against the fp32 product."""
    g = torch.Generator().manual_seed(0)
    w = torch.randn(n, 1024, generator=g) * 0.02
    lin = Int8IslandLinear.from_dense("x", w, "cuda")
    assert lin._gemm is not None
    for M in (1, 7, 300):
        x = torch.randn(M, 1024, generator=g).bfloat16()
        y = lin(x.cuda())
        torch.cuda.synchronize()
        assert ops.status() == 0
        ref = (x.float() @ (lin.q.float().cpu() * lin.scale.float().cpu()[:, None]).t())
        assert (y.float().cpu() - ref).abs().max().item() <= 1e-2 * ref.abs().max().item() + 1e-3


@pytest.mark.parametrize("w4a8", ["w4a16", "w4a8"])
def test_forward_with_island_layer_matches_reference(w4a8, monkeypatch):
    monkeypatch.setenv("K8V4_PREFILL_GEMM", w4a8)
    dev = torch.device("cuda")
    m = DenseModel(TINY, device=dev).random_init(seed=3)
    L = m.layers[1]
    for f in ("qkv", "o", "gate_up", "down"):
        lin = getattr(L, f)
        dense = gptq.dequant_int4(lin.qweight, lin.scales).t().contiguous()
        setattr(L, f, Int8IslandLinear.from_dense(lin.name, dense, dev))
    prompts = [list(range(3, 3 + 150)), list(range(100, 100 + 45))]
    inp = _inputs(prompts, lambda i: 2 * i + 1, dev)
    caches = [torch.zeros(64, m.layout.page_bytes, dtype=torch.uint8, device=dev) for _ in m.layers]
    out = m.forward(inp, caches)
    torch.cuda.synchronize()
    assert ops.status() == 0
    ref_caches = [torch.zeros(64, m.layout.page_bytes, dtype=torch.uint8) for _ in m.layers]
    ref = m.reference_forward(inp, ref_caches)
    err = (out.float().cpu() - ref.float()).abs().max().item()
    scale = ref.float().abs().max().item()
    tol = 0.06 if w4a8 == "w4a8" else 0.03
    assert err <= tol * scale, (err, scale)
