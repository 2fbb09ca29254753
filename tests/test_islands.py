"""INT8 islands: suffix selection, the quantization rule, dense-weight loading
with TP sharding (CPU). Behaviour of the reference's ``int8_island.py``."""
import torch
from safetensors.torch import save_file

from k8v4_xpu_b200.layers.linear import Int4Linear, Int8IslandLinear, is_island, island_suffixes
from k8v4_xpu_b200.models import gptq
from k8v4_xpu_b200.models.checkpoint import load_checkpoint, save_checkpoint
from k8v4_xpu_b200.models.config import TINY
from k8v4_xpu_b200.models.dense import DenseModel


def test_suffix_list_and_matching():
    env = {"K8V4_INT8_ISLANDS": " layers.1.self_attn.qkv_proj, mlp.down_proj ,,"}
    suf = island_suffixes(env)
    assert suf == ("layers.1.self_attn.qkv_proj", "mlp.down_proj")
    assert is_island("model.layers.1.self_attn.qkv_proj", suf)
    assert not is_island("model.layers.11.self_attn.o_proj", suf)
    assert is_island("model.layers.0.mlp.down_proj", suf)
    assert island_suffixes({}) == ()


def test_quantize_rule_matches_reference_formula():
    g = torch.Generator().manual_seed(0)
    w = torch.randn(64, 256, generator=g)
    w[3] = 0.0  # an all-zero row keeps the 1e-12 floor
    q, s = Int8IslandLinear.quantize(w)
    ref_s = (w.abs().amax(1, keepdim=True) / 127.0).clamp_min(1e-12)
    ref_q = torch.round(w / ref_s).clamp(-127, 127).to(torch.int8)
    assert torch.equal(q, ref_q)
    assert torch.allclose(s.float(), ref_s.reshape(-1).bfloat16().float())
    assert q.abs().max().item() == 127 and q[3].abs().max().item() == 0
    lin = Int8IslandLinear("x", q, s)
    x = torch.randn(5, 256, generator=g)
    err = (lin.reference(x) - x @ w.t()).abs().max().item()
    assert err < 0.02 * (x @ w.t()).abs().max().item()


def _dense_from_gptq(lin):
    return gptq.dequant_int4(lin.qweight, lin.scales).t().contiguous()  # [N, K]


def _write_dense(m, path, layer):
    """Add dense HF weights of one layer's linears (exact dequantized int4)."""
    L = m.layers[layer]
    cfg = m.cfg
    pre = "model.layers.%d." % layer
    qkv = _dense_from_gptq(L.qkv)
    q_sz, kv_sz = cfg.q_size, cfg.kv_size
    gu = _dense_from_gptq(L.gate_up)
    I = cfg.intermediate
    t = {pre + "self_attn.q_proj.weight": qkv[:q_sz], pre + "self_attn.k_proj.weight": qkv[q_sz:q_sz + kv_sz],
         pre + "self_attn.v_proj.weight": qkv[q_sz + kv_sz:], pre + "self_attn.o_proj.weight": _dense_from_gptq(L.o),
         pre + "mlp.gate_proj.weight": gu[:I], pre + "mlp.up_proj.weight": gu[I:],
         pre + "mlp.down_proj.weight": _dense_from_gptq(L.down)}
    save_file({k: v.bfloat16().contiguous() for k, v in t.items()}, str(path / "islands.safetensors"))


def test_islands_load_from_dense_weights_and_shard(tmp_path, monkeypatch):
    full = DenseModel(TINY, device="cpu").random_init(seed=3)
    save_checkpoint(full, str(tmp_path))
    _write_dense(full, tmp_path, 1)
    monkeypatch.setenv("K8V4_INT8_ISLANDS", "layers.1.self_attn.qkv_proj,layers.1.self_attn.o_proj,"
                                            "layers.1.mlp.gate_up_proj,layers.1.mlp.down_proj")
    g = torch.Generator().manual_seed(1)
    for tp in (1, 2):
        for rank in range(tp):
            ref = DenseModel(TINY, tp=tp, rank=rank, device="cpu").random_init(seed=3)
            m = DenseModel(TINY, tp=tp, rank=rank, device="cpu")
            load_checkpoint(m, str(tmp_path))
            assert isinstance(m.layers[0].qkv, Int4Linear)
            for f in ("qkv", "o", "gate_up", "down"):
                isl, gl = getattr(m.layers[1], f), getattr(ref.layers[1], f)
                assert isinstance(isl, Int8IslandLinear), f
                assert (isl.out_features, isl.in_features) == (gl.out_features, gl.in_features), f
                x = torch.randn(3, gl.in_features, generator=g)
                want = gl.reference(x)
                err = (isl.reference(x) - want).abs().max().item()
                assert err < 0.02 * want.abs().max().item() + 1e-4, (tp, rank, f, err)
