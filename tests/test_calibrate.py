"""Live-model GPTQ calibration hooks (CPU): Hessians of every quantized linear,
held-out rows, TP gathers of row-parallel inputs, and the bake consuming them."""
import json
import os
import socket
import traceback

import pytest
import torch
import torch.multiprocessing as mp

from k8v4_xpu_b200.layers.linear import Int4Linear
from k8v4_xpu_b200.models.config import TINY
from k8v4_xpu_b200.models.dense import DenseModel
from k8v4_xpu_b200.tools import bake
from k8v4_xpu_b200.tools.calibrate import Calibrator, checkpoint_names

ONE_LAYER = TINY.__class__(**{**TINY.__dict__, "num_layers": 1})


def _cpu_linear(self, x=None, xq=None, xs=None, **kw):
    """A CPU stand-in for the tcgen05 GEMM: the dequantized weight product."""
    a = x.float() if x is not None else xq.float() * xs.float().view(-1, 1)
    return (a @ self.dense_t()).bfloat16()


def _fake_forward(m, rows, gen):
    """Drive every linear of the model once, as a forward would."""
    cfg = m.cfg
    seen = {}
    for li, L in enumerate(m.layers + [m.mtp.layer]):
        x = torch.randn(rows, cfg.hidden, generator=gen).bfloat16()
        L.qkv(x)
        a = torch.randn(rows, L.o.in_features, generator=gen).bfloat16()
        L.o(a)
        L.gate_up(x)
        act = torch.randn(rows, L.down.in_features, generator=gen)
        q = torch.clamp(torch.round(act * 20), -127, 127).to(torch.int8)
        s = torch.full((rows,), 0.05)
        L.down(xq=q, xs=s)  # the W4A8 path: int8 codes and per-row scales
        seen[li] = (x, a, q.float() * 0.05)
    cat = torch.randn(rows, 2 * cfg.hidden, generator=gen).bfloat16()
    m.mtp.eh_proj(cat)
    return seen, cat


def _kept(x, every=64):
    idx = torch.arange(x.shape[0])
    return x[(idx % every) != every - 1].double()


def test_calibrator_collects_every_linear_with_held_out_rows(monkeypatch, tmp_path):
    monkeypatch.setattr(Int4Linear, "__call__", _cpu_linear)
    m = DenseModel(ONE_LAYER, device="cpu").random_init(seed=3)
    m.init_mtp(seed=4)
    originals = (m.layers[0].qkv, m.layers[0].down, m.mtp.eh_proj)
    calib = Calibrator(m).attach()
    assert isinstance(m.layers[0].qkv, Int4Linear) and m.layers[0].qkv is not originals[0]
    gen = torch.Generator().manual_seed(0)
    rows = 130
    seen, cat = _fake_forward(m, rows, gen)
    calib.detach()
    assert (m.layers[0].qkv, m.layers[0].down, m.mtp.eh_proj) == originals
    H = calib.hessians()
    per_layer = ("self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj", "self_attn.o_proj",
                 "mlp.gate_proj", "mlp.up_proj", "mlp.down_proj")
    want = {"model.layers.0." + n for n in per_layer} | {"mtp.layers.0." + n for n in per_layer} | {"mtp.eh_proj"}
    assert set(H) == want
    x, a, act = seen[0]
    kx, ka, kact = _kept(x.float()), _kept(a.float()), _kept(act)
    assert torch.allclose(H["model.layers.0.self_attn.q_proj"], 2 * kx.t() @ kx / kx.shape[0], rtol=1e-5, atol=1e-6)
    assert H["model.layers.0.self_attn.k_proj"] is H["model.layers.0.self_attn.q_proj"]  # one shared input
    assert torch.allclose(H["model.layers.0.self_attn.o_proj"], 2 * ka.t() @ ka / ka.shape[0], rtol=1e-5, atol=1e-6)
    assert torch.allclose(H["model.layers.0.mlp.down_proj"], 2 * kact.t() @ kact / kact.shape[0], rtol=1e-5,
                          atol=1e-6)
    kc = _kept(cat.float())
    assert torch.allclose(H["mtp.eh_proj"], 2 * kc.t() @ kc / kc.shape[0], rtol=1e-5, atol=1e-6)
    # rows 63 and 127 of the 130 were held out of the statistics and kept aside
    held = calib.heldout_inputs("model.layers.0.self_attn.o_proj")
    assert held.shape[0] == 2 and torch.equal(held, a.float()[[63, 127]])
    # the output error of a quantized weight on the held-out rows
    w = torch.randn(ONE_LAYER.hidden, 256, generator=gen) * 0.02
    name = "model.layers.0.mlp.gate_proj"
    deq = lambda c, s: ((c.float() - 8).view(-1, 128, 256) * s.view(-1, 1, 256)).view(-1, 256)  # noqa: E731
    wq = deq(*bake.gptq_quantize(w, H[name]))
    hx = x.float()[[63, 127]].double()
    err = float(((hx @ (w.double() - wq.double())) ** 2).sum() / 2)
    assert abs(calib.heldout_error(name, w, wq) - err) <= 1e-9 * max(1.0, err)
    # saved atomically, then consumed by the bake
    path = calib.save(str(tmp_path / "hessians.pt"))
    assert not os.path.exists(path + ".partial")
    loaded = torch.load(path)
    assert set(loaded) == want and torch.equal(loaded["mtp.eh_proj"], H["mtp.eh_proj"])


def test_select_limits_the_taps_and_names_map_back():
    assert checkpoint_names("model.layers.3.mlp.gate_up_proj") == ("model.layers.3.mlp.gate_proj",
                                                                  "model.layers.3.mlp.up_proj")
    assert checkpoint_names("mtp.eh_proj") == ("mtp.eh_proj",)
    m = DenseModel(ONE_LAYER, device="cpu").random_init(seed=3)
    m.init_mtp(seed=4)
    with Calibrator(m, select=r"^mtp\.") as calib:
        assert type(m.layers[0].qkv) is Int4Linear  # not tapped
        assert type(m.mtp.layer.qkv) is not Int4Linear
    assert type(m.mtp.layer.qkv) is Int4Linear
    assert calib.hessians() == {}
    with pytest.raises(ValueError):
        Calibrator(m, holdout_every=1)


def test_bake_consumes_collected_hessians(monkeypatch, tmp_path):
    from safetensors.torch import save_file
    from k8v4_xpu_b200.models.checkpoint import config_to_hf
    monkeypatch.setattr(Int4Linear, "__call__", _cpu_linear)
    src, out = tmp_path / "dense", tmp_path / "gptq"
    src.mkdir()
    cfg = ONE_LAYER
    hf = config_to_hf(cfg)
    hf.pop("quantization_config")
    (src / "config.json").write_text(json.dumps(hf))
    g = torch.Generator().manual_seed(1)
    H_, I_ = cfg.hidden, cfg.intermediate
    dims = {"self_attn.q_proj": (cfg.q_size, H_), "self_attn.k_proj": (cfg.kv_size, H_),
            "self_attn.v_proj": (cfg.kv_size, H_), "self_attn.o_proj": (H_, cfg.q_size),
            "mlp.gate_proj": (I_, H_), "mlp.up_proj": (I_, H_), "mlp.down_proj": (H_, I_)}
    t = {"model.layers.0.%s.weight" % k: (torch.randn(*s, generator=g) * 0.02).bfloat16() for k, s in dims.items()}
    for nm in ("input_layernorm", "post_attention_layernorm"):
        t["model.layers.0.%s.weight" % nm] = torch.ones(H_).bfloat16()
    t["model.norm.weight"] = torch.ones(H_).bfloat16()
    t["model.embed_tokens.weight"] = (torch.randn(cfg.vocab, H_, generator=g) * 0.02).bfloat16()
    save_file(t, str(src / "model.safetensors"))
    m = DenseModel(cfg, device="cpu").random_init(seed=3)
    m.init_mtp(seed=4)
    with Calibrator(m, select=r"^model\.") as calib:
        _fake_forward(m, 200, torch.Generator().manual_seed(2))
    rep = bake.bake_dense(str(src), str(out), hessians=torch.load(calib.save(str(tmp_path / "h.pt"))))
    assert rep == {"linears_gptq": 7, "linears_rtn": 0, "layers": 1}


def _port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _tp_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    import torch.distributed as dist
    try:
        from k8v4_xpu_b200.parallel.comm import TPComm, init_from_env
        init_from_env(timeout_s=60, backend="gloo")
        Int4Linear.__call__ = _cpu_linear
        m = DenseModel(ONE_LAYER, tp=world, rank=rank, device="cpu", comm=TPComm()).random_init(seed=3)
        gen = torch.Generator().manual_seed(9)  # the same full inputs on every rank
        x = torch.randn(70, ONE_LAYER.hidden, generator=gen).bfloat16()
        a_full = torch.randn(70, ONE_LAYER.q_size, generator=gen).bfloat16()
        k = a_full.shape[1] // world
        with Calibrator(m) as calib:
            m.layers[0].qkv(x)  # column-parallel: every rank sees the whole input
            m.layers[0].o(a_full[:, rank * k:(rank + 1) * k])  # row-parallel: this rank's K slice
        H = calib.hessians()
        # numpy arrays travel by value (tensors would share memory with a process that exits)
        q.put((rank, {"qkv": H["model.layers.0.self_attn.q_proj"].numpy(),
                      "o": H["model.layers.0.self_attn.o_proj"].numpy(),
                      "x": x.float().numpy(), "a": a_full.float().numpy()}))
    except Exception:
        q.put((rank, {"error": traceback.format_exc()}))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


def test_row_parallel_inputs_are_gathered_across_tp_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_tp_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    out = dict(q.get(timeout=180) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    for r in range(2):
        assert "error" not in out[r], out[r]["error"]
    out = {r: ({k: torch.from_numpy(v) for k, v in o.items()}) for r, o in out.items()}
    ka, kx = _kept(out[0]["a"]), _kept(out[0]["x"])
    for r in range(2):
        assert out[r]["o"].shape == (ONE_LAYER.q_size, ONE_LAYER.q_size)  # full K, not the shard
        assert torch.allclose(out[r]["o"], 2 * ka.t() @ ka / ka.shape[0], rtol=1e-5, atol=1e-6)
        assert torch.allclose(out[r]["qkv"], 2 * kx.t() @ kx / kx.shape[0], rtol=1e-5, atol=1e-6)
