"""Offline checkpoint tools (the reference's bake pipeline, T4-T8).

* ``gptq_quantize``: GPTQ int4 (group 128, symmetric) of one linear from its
  input Hessian ``H = 2 X^T X / n`` (Frantar et al., 2022, "GPTQ: Accurate
  Post-Training Quantization for Generative Pre-trained Transformers",
  Algorithm 1): columns are quantized in order and each column's error is
  propagated to the not-yet-quantized columns through the upper Cholesky
  factor of ``H^-1``; a group's scale (``amax / 7``, stored fp16) is fixed when
  the group starts. Without a Hessian it is round-to-nearest.
* ``HessianAccumulator``: running ``X^T X`` of a linear's inputs (the
  calibration hooks of ``tools/calibrate_swift_bake.py``).
* ``bake_dense``: a dense HF-style checkpoint (bf16 ``[out, in]`` linears) to
  the GPTQ + INT8 side-file format (``bake_gptq_resume.py`` +
  ``assemble_swift_bake.py``).
* ``random_checkpoint``: random-init weights of a preset, written in the
  same format (the checkpoint the benchmarks load when no real one exists).
* ``verify_checkpoint``: every linear present, shapes consistent, symmetric
  zeros, no act-order (``prepare_swift_autoround.py``).

    python -m k8v4_xpu_b200.tools.bake random --preset tiny --out DIR
    python -m k8v4_xpu_b200.tools.bake dense --src DIR --out DIR [--hessians FILE]
    python -m k8v4_xpu_b200.tools.bake verify DIR
"""
from __future__ import annotations

import argparse
import glob
import json
import os
import sys

import torch

from ..models import gptq
from ..models.checkpoint import SIDE_FILE, _linear_tensors, _save, _save_json, config_from_hf, config_to_hf

LINEARS = ("self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj", "self_attn.o_proj", "mlp.gate_proj",
           "mlp.up_proj", "mlp.down_proj")


def gptq_quantize(w_kn: torch.Tensor, H: torch.Tensor | None = None, group: int = 128,
                  damp: float = 0.01) -> tuple[torch.Tensor, torch.Tensor]:
    """Quantize ``w`` laid out ``[K, N]``; returns (codes uint8 [K, N], scales fp32 [K/group, N])."""
    if H is None:
        return gptq.quantize_int4_rtn(w_kn, group)
    K, N = w_kn.shape
    if K % group:
        raise ValueError("K must be a multiple of %d" % group)
    W = w_kn.t().double().clone()          # [N, K]: one row per output feature
    H = H.double().clone()
    dead = torch.diag(H) == 0
    H[dead, dead] = 1.0
    W[:, dead] = 0.0
    H += damp * torch.mean(torch.diag(H)) * torch.eye(K, dtype=H.dtype)
    U = torch.linalg.cholesky(torch.cholesky_inverse(torch.linalg.cholesky(H)), upper=True)
    codes = torch.zeros((N, K), dtype=torch.uint8)
    scales = torch.zeros((K // group, N), dtype=torch.float32)
    for g0 in range(0, K, group):
        s = (W[:, g0:g0 + group].abs().amax(dim=1).clamp_min(1e-9) / 7.0).half().double()
        scales[g0 // group] = s.float()
        for i in range(g0, g0 + group):
            w = W[:, i]
            q = torch.clamp(torch.round(w / s), -8, 7)
            codes[:, i] = (q + 8).to(torch.uint8)
            err = (w - q * s) / U[i, i]
            W[:, i + 1:] -= err.unsqueeze(1) * U[i, i + 1:].unsqueeze(0)
    return codes.t().contiguous(), scales


class HessianAccumulator:
    """``2 X^T X / n`` over calibration rows ``x`` [rows, K] of one linear."""

    def __init__(self, k: int):
        self.H = torch.zeros((k, k), dtype=torch.float64)
        self.n = 0

    def add(self, x: torch.Tensor) -> None:
        x = x.reshape(-1, x.shape[-1]).double().cpu()
        m = x.shape[0]
        self.H *= self.n / (self.n + m)
        self.n += m
        x = x * (2.0 / self.n) ** 0.5
        self.H += x.t() @ x


def _dense_tensors(src: str) -> dict:
    from safetensors import safe_open
    out = {}
    for fn in sorted(glob.glob(os.path.join(src, "*.safetensors"))):
        with safe_open(fn, framework="pt") as h:
            for k in h.keys():
                out[k] = h.get_tensor(k)
    return out


def bake_dense(src: str, out: str, hessians: dict | None = None, layers: int | None = None) -> dict:
    """Quantize a dense checkpoint into the GPTQ + side-file format. Returns a summary."""
    with open(os.path.join(src, "config.json")) as f:
        hf = json.load(f)
    hf.pop("quantization_config", None)
    cfg = config_from_hf(hf)
    t = _dense_tensors(src)
    os.makedirs(out, exist_ok=True)
    shard: dict = {}
    n_gptq = n_rtn = 0
    L = cfg.num_layers if layers is None else layers
    prefixes = ["model.layers.%d." % i for i in range(L)]
    if any(k.startswith("mtp.") for k in t):
        prefixes.append("mtp.layers.0.")
    for pre in prefixes:
        for lin in LINEARS:
            name = pre + lin
            w = t[name + ".weight"].float().t().contiguous()  # [K, N]
            H = hessians.get(name) if hessians else None
            codes, scales = gptq_quantize(w, H)
            n_gptq += H is not None
            n_rtn += H is None
            packed = gptq.pack_int4(codes, scales)
            shard.update(_linear_tensors(name, packed["qweight"], packed["scales"]))
        for norm in ("input_layernorm.weight", "post_attention_layernorm.weight"):
            shard[pre + norm] = t[pre + norm].to(torch.bfloat16)
    if "mtp.eh_proj.weight" in t:
        codes, scales = gptq_quantize(t["mtp.eh_proj.weight"].float().t().contiguous(),
                                      hessians.get("mtp.eh_proj") if hessians else None)
        packed = gptq.pack_int4(codes, scales)
        shard.update(_linear_tensors("mtp.eh_proj", packed["qweight"], packed["scales"]))
        for n in ("mtp.enorm.weight", "mtp.hnorm.weight", "mtp.norm.weight"):
            shard[n] = t[n].to(torch.bfloat16)
    shard["model.norm.weight"] = t["model.norm.weight"].to(torch.bfloat16)
    head = t.get("lm_head.weight", t["model.embed_tokens.weight"])
    hq, hs = gptq.quantize_int8_rows(head.float())
    shard["lm_head.weight"], shard["lm_head.weight_scale"] = hq, hs
    _save(shard, os.path.join(out, "model-00000.safetensors"))
    eq, es = gptq.quantize_int8_rows(t["model.embed_tokens.weight"].float())
    _save({"embed_tokens.int8": eq, "embed_tokens.scale": es}, os.path.join(out, SIDE_FILE))
    new_cfg = config_to_hf(cfg if layers is None else cfg.__class__(**{**cfg.__dict__, "num_layers": L}))
    _save_json(new_cfg, os.path.join(out, "config.json"))  # last: the directory is complete
    return {"linears_gptq": n_gptq, "linears_rtn": n_rtn, "layers": L}


def random_checkpoint(out: str, preset: str = "tiny", layers: int | None = None, seed: int = 0, mtp: bool = True,
                      device: str = "cpu") -> str:
    from ..models.checkpoint import save_checkpoint
    from ..models.config import PRESETS
    from ..models.dense import DenseModel
    cfg = PRESETS[preset]
    if layers is not None:
        cfg = cfg.__class__(**{**cfg.__dict__, "num_layers": layers})
    m = DenseModel(cfg, device=device).random_init(seed=seed)
    if mtp:
        m.init_mtp(seed=seed)
    save_checkpoint(m, out)
    return out


def verify_checkpoint(path: str) -> dict:
    """Check a GPTQ checkpoint's linears; returns a report, raises on a problem."""
    from ..models.checkpoint import _Reader, read_model_config
    cfg = read_model_config(path)
    r = _Reader(path)
    n = 0
    shapes = {"self_attn.q_proj": (cfg.hidden, cfg.q_size), "self_attn.k_proj": (cfg.hidden, cfg.kv_size),
              "self_attn.v_proj": (cfg.hidden, cfg.kv_size), "self_attn.o_proj": (cfg.q_size, cfg.hidden),
              "mlp.gate_proj": (cfg.hidden, cfg.intermediate), "mlp.up_proj": (cfg.hidden, cfg.intermediate),
              "mlp.down_proj": (cfg.intermediate, cfg.hidden)}
    for i in range(cfg.num_layers):
        for lin, (k, nn) in shapes.items():
            qw, sc = r.linear("model.layers.%d.%s" % (i, lin))
            if tuple(qw.shape) != (k // 8, nn) or tuple(sc.shape) != (k // 128, nn):
                raise ValueError("layer %d %s: qweight %s scales %s" % (i, lin, tuple(qw.shape), tuple(sc.shape)))
            n += 1
    return {"layers": cfg.num_layers, "linears": n, "mtp": r.has("mtp.eh_proj.qweight"),
            "lm_head_rows": int(r.get("lm_head.weight").shape[0])}


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="k8v4-bake")
    sub = ap.add_subparsers(dest="cmd", required=True)
    a = sub.add_parser("random")
    a.add_argument("--preset", default="tiny")
    a.add_argument("--layers", type=int)
    a.add_argument("--seed", type=int, default=0)
    a.add_argument("--no-mtp", action="store_true")
    a.add_argument("--device", default="cpu")
    a.add_argument("--out", required=True)
    d = sub.add_parser("dense")
    d.add_argument("--src", required=True)
    d.add_argument("--out", required=True)
    d.add_argument("--hessians", help="torch file: {linear name: H [K, K]}")
    v = sub.add_parser("verify")
    v.add_argument("path")
    args = ap.parse_args(argv)
    if args.cmd == "random":
        random_checkpoint(args.out, args.preset, args.layers, args.seed, not args.no_mtp, args.device)
        print(json.dumps(verify_checkpoint(args.out)))
    elif args.cmd == "dense":
        H = torch.load(args.hessians) if args.hessians else None
        print(json.dumps(bake_dense(args.src, args.out, H)))
    else:
        print(json.dumps(verify_checkpoint(args.path)))
    return 0


if __name__ == "__main__":
    sys.exit(main())
