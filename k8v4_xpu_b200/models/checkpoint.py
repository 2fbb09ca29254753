"""GPTQ INT4 + INT8 side-file checkpoints: read, write, load with TP sharding.

On-disk format (the reference's baked checkpoint, ``tools/bake_gptq_resume.py
:51-75``, ``tools/assemble_swift_bake.py:58-147`` with the side-file entry at
``:118,135``, read back by ``k8v4_v030/embed_int8_runtime.py:20-50``):

* ``config.json``: HF-style architecture keys, ``quantization_config``
  (``quant_method: gptq, bits: 4, group_size: 128, sym: true, desc_act:
  false``) and ``embed_tokens_quant`` (``bits: 8, side_file, key_weight,
  key_scale``);
* ``model.safetensors`` (or ``model-*.safetensors`` shards): per linear
  ``<name>.qweight`` int32 ``[K/8, N]``, ``.scales`` fp16 ``[K/128, N]``,
  ``.qzeros`` int32 ``[K/128, N/8]`` (0x77777777), ``.g_idx`` int32 ``[K]``;
  norms in bf16; the lm_head as per-row int8 ``lm_head.weight`` +
  ``lm_head.weight_scale``;
* the side file (``embed_int8.safetensors``): int8 codes ``[V, H]`` and fp16
  scales ``[V, 1]`` of the embedding.

Linear names follow the HF layout (``self_attn.{q,k,v,o}_proj``,
``mlp.{gate,up,down}_proj``); the loader fuses q|k|v and gate|up into this
framework's column-parallel projections and keeps only this rank's shard
(the embedding side file materializes only the rank's vocab rows, like
``embed_int8_runtime.py:11-50``).
"""
from __future__ import annotations

import glob
import json
import os

import torch

from . import gptq
from .config import ModelConfig

SIDE_FILE = "embed_int8.safetensors"


def config_to_hf(cfg: ModelConfig) -> dict:
    return {
        "architectures": ["K8V4DenseForCausalLM"], "model_type": "k8v4_dense", "name": cfg.name,
        "hidden_size": cfg.hidden, "num_hidden_layers": cfg.num_layers, "num_attention_heads": cfg.num_heads,
        "num_key_value_heads": cfg.num_kv_heads, "head_dim": cfg.head_dim, "intermediate_size": cfg.intermediate,
        "vocab_size": cfg.vocab, "rms_norm_eps": cfg.rms_eps, "rope_theta": cfg.rope_theta,
        "max_position_embeddings": cfg.max_position, "num_nextn_predict_layers": cfg.mtp_layers,
        "torch_dtype": "bfloat16",
        "quantization_config": {"quant_method": "gptq", "bits": 4, "group_size": cfg.group_size, "sym": True,
                                "desc_act": False, "lm_head": "int8_per_row"},
        "embed_tokens_quant": {"bits": 8, "side_file": SIDE_FILE, "key_weight": "embed_tokens.int8",
                               "key_scale": "embed_tokens.scale"},
    }


def config_from_hf(d: dict) -> ModelConfig:
    q = d.get("quantization_config", {})
    if q and (q.get("quant_method") != "gptq" or q.get("bits") != 4 or not q.get("sym", True)
              or q.get("desc_act", False)):
        raise ValueError("expected symmetric GPTQ int4 without act-order, got %r" % q)
    return ModelConfig(
        name=d.get("name", d.get("model_type", "checkpoint")), num_layers=d["num_hidden_layers"],
        hidden=d["hidden_size"], num_heads=d["num_attention_heads"], num_kv_heads=d["num_key_value_heads"],
        head_dim=d.get("head_dim", d["hidden_size"] // d["num_attention_heads"]),
        intermediate=d["intermediate_size"], vocab=d["vocab_size"], rms_eps=d.get("rms_norm_eps", 1e-6),
        rope_theta=d.get("rope_theta", 1e6), max_position=d.get("max_position_embeddings", 262144 + 8192),
        group_size=q.get("group_size", 128), mtp_layers=d.get("num_nextn_predict_layers", 0))


def read_model_config(path: str) -> ModelConfig:
    with open(os.path.join(path, "config.json")) as f:
        return config_from_hf(json.load(f))


def _save(tensors: dict, path: str) -> None:
    """Atomic: written to ``path.partial``, then renamed over ``path``."""
    from safetensors.torch import save_file
    tmp = path + ".partial"
    save_file({k: v.contiguous().cpu() for k, v in tensors.items()}, tmp)
    os.replace(tmp, path)


def _save_json(obj, path: str, indent: int = 2) -> None:
    tmp = path + ".partial"
    with open(tmp, "w") as f:
        json.dump(obj, f, indent=indent)
    os.replace(tmp, path)


def _linear_tensors(prefix: str, qweight: torch.Tensor, scales: torch.Tensor) -> dict:
    K8, N = qweight.shape
    groups = scales.shape[0]
    return {prefix + ".qweight": qweight, prefix + ".scales": scales.half(),
            prefix + ".qzeros": torch.full((groups, max(1, N // 8)), gptq.QZERO_WORD, dtype=torch.int32),
            prefix + ".g_idx": torch.arange(K8 * 8, dtype=torch.int32) // 128}


def save_checkpoint(model, path: str, shard_layers: int = 8) -> None:
    """Write a TP1 ``DenseModel`` in the GPTQ + side-file format (HF names,
    q/k/v and gate/up unfused).

    Every file is written atomically (``.partial``, then renamed; the
    reference's bake tools do the same, ``tools/assemble_swift_bake.py:41-55``, ``tools/calibrate_swift_bake.py:105-106``)
    and ``config.json`` comes last, so a directory holding one is complete."""
    if model.tp != 1:
        raise ValueError("save a tensor-parallel size 1 model")
    from ..layers.linear import Int4Linear
    if any(not isinstance(lin, Int4Linear) for L in model.layers for lin in (L.qkv, L.o, L.gate_up, L.down)):
        raise ValueError("INT8 islands are chosen when loading (K8V4_INT8_ISLANDS); save the GPTQ model")
    cfg = model.cfg
    os.makedirs(path, exist_ok=True)
    q_sz, kv_sz = cfg.q_size, cfg.kv_size
    shard: dict = {}
    idx = 0
    index = {"weight_map": {}}

    def flush(final=False):
        nonlocal shard, idx
        if shard and (final or len(shard) >= 40 * shard_layers):
            name = "model-%05d.safetensors" % idx
            _save(shard, os.path.join(path, name))
            for k in shard:
                index["weight_map"][k] = name
            shard, idx = {}, idx + 1

    def put_layer(pre: str, L) -> None:
        qw, sc = L.qkv.qweight.cpu(), L.qkv.scales.cpu()
        for nm, a, b in (("q_proj", 0, q_sz), ("k_proj", q_sz, q_sz + kv_sz), ("v_proj", q_sz + kv_sz,
                                                                                 q_sz + 2 * kv_sz)):
            shard.update(_linear_tensors(pre + "self_attn." + nm, qw[:, a:b], sc[:, a:b]))
        shard.update(_linear_tensors(pre + "self_attn.o_proj", L.o.qweight.cpu(), L.o.scales.cpu()))
        gw, gs = L.gate_up.qweight.cpu(), L.gate_up.scales.cpu()
        I = cfg.intermediate
        shard.update(_linear_tensors(pre + "mlp.gate_proj", gw[:, :I], gs[:, :I]))
        shard.update(_linear_tensors(pre + "mlp.up_proj", gw[:, I:], gs[:, I:]))
        shard.update(_linear_tensors(pre + "mlp.down_proj", L.down.qweight.cpu(), L.down.scales.cpu()))
        shard[pre + "input_layernorm.weight"] = L.input_norm.cpu()
        shard[pre + "post_attention_layernorm.weight"] = L.post_norm.cpu()

    for i, L in enumerate(model.layers):
        put_layer("model.layers.%d." % i, L)
        flush()
    if model.mtp is not None:
        M = model.mtp
        put_layer("mtp.layers.0.", M.layer)
        shard.update(_linear_tensors("mtp.eh_proj", M.eh_proj.qweight.cpu(), M.eh_proj.scales.cpu()))
        shard["mtp.enorm.weight"] = M.enorm.cpu()
        shard["mtp.hnorm.weight"] = M.hnorm.cpu()
        shard["mtp.norm.weight"] = M.norm.cpu()
    shard["model.norm.weight"] = model.final_norm.cpu()
    lm = model.lm_head
    shard["lm_head.weight"] = lm.weight[: lm.out_features].cpu()
    shard["lm_head.weight_scale"] = lm.scale[: lm.out_features].view(-1, 1).cpu()
    flush(final=True)
    _save_json(index, os.path.join(path, "model.safetensors.index.json"), indent=1)
    _save({"embed_tokens.int8": model.embed_codes.cpu(), "embed_tokens.scale": model.embed_scales.view(-1, 1).cpu()},
          os.path.join(path, SIDE_FILE))
    _save_json(config_to_hf(cfg), os.path.join(path, "config.json"))


class _Reader:
    """Lazy tensor access over every ``*.safetensors`` of a checkpoint."""

    def __init__(self, path: str):
        from safetensors import safe_open
        self.files = {}
        for fn in sorted(glob.glob(os.path.join(path, "*.safetensors"))):
            if os.path.basename(fn) == SIDE_FILE:
                continue
            h = safe_open(fn, framework="pt")
            for k in h.keys():
                self.files[k] = h

    def get(self, name: str) -> torch.Tensor:
        if name not in self.files:
            raise KeyError("checkpoint has no tensor %r" % name)
        return self.files[name].get_tensor(name)

    def has(self, name: str) -> bool:
        return name in self.files

    def linear(self, prefix: str) -> tuple[torch.Tensor, torch.Tensor]:
        qw, sc = self.get(prefix + ".qweight"), self.get(prefix + ".scales")
        if self.has(prefix + ".qzeros"):
            qz = self.get(prefix + ".qzeros")
            if not bool((qz == gptq.QZERO_WORD).all()):
                raise ValueError("%s: only symmetric GPTQ (qzeros 0x77777777) is supported" % prefix)
        if self.has(prefix + ".g_idx"):
            g = self.get(prefix + ".g_idx")
            if not torch.equal(g, torch.arange(g.numel(), dtype=g.dtype) // 128):
                raise ValueError("%s: act-order (permuted g_idx) is not supported" % prefix)
        return qw, sc


def _rows_k(wt: torch.Tensor, rank: int, k_local: int) -> torch.Tensor:
    """Row-parallel shard of a dense [K, N] weight: this rank's K rows."""
    return wt[rank * k_local:(rank + 1) * k_local]


def load_checkpoint(model, path: str) -> None:
    """Load a GPTQ + side-file checkpoint into ``model`` (its TP rank's shard).

    Linears whose fused module name ends with a ``K8V4_INT8_ISLANDS`` suffix
    are read from dense ``<part>.weight`` tensors instead and kept as INT8
    islands."""
    from ..layers.linear import Int4Linear, Int8IslandLinear, Int8RowLinear, is_island, island_suffixes
    from .dense import LayerWeights, MTPWeights, rope_table
    cfg = read_model_config(path)
    mc = model.cfg
    for f in ("hidden", "num_heads", "num_kv_heads", "head_dim", "intermediate", "vocab"):
        if getattr(cfg, f) != getattr(mc, f):
            raise ValueError("checkpoint %s=%s does not match the model's %s" % (f, getattr(cfg, f),
                                                                                getattr(mc, f)))
    dev = model.device
    r = _Reader(path)
    sh = model.shape

    islands = island_suffixes()

    def dense_t(pre: str, parts) -> torch.Tensor:
        # dense HF weights [N_part, K] of the parts, fused along N, as [K, N]
        return torch.cat([r.get(pre + "%s.weight" % p).float() for p in parts], 0).t()

    def island(mod: str, wt_local: torch.Tensor) -> Int8IslandLinear:
        return Int8IslandLinear.from_dense(mod, wt_local.t().contiguous(), dev)

    def layer(pre: str, name: str) -> LayerWeights:
        # INT8 islands (K8V4_INT8_ISLANDS suffixes of the fused module names)
        # come from dense weights, quantized per output row after sharding
        qkv_name, o_name = name + "self_attn.qkv_proj", name + "self_attn.o_proj"
        gu_name, dn_name = name + "mlp.gate_up_proj", name + "mlp.down_proj"
        if is_island(qkv_name, islands):
            wt = dense_t(pre + "self_attn.", ("q_proj", "k_proj", "v_proj"))
            qkv = island(qkv_name, model._shard_qkv(wt, wt[:1])[0])
        else:
            qs = [r.linear(pre + "self_attn.%s_proj" % p) for p in ("q", "k", "v")]
            qkv_q, qkv_s = model._shard_qkv(torch.cat([a for a, _ in qs], 1), torch.cat([b for _, b in qs], 1))
            qkv = Int4Linear(qkv_name, qkv_q.to(dev).contiguous(), qkv_s.to(dev).contiguous())
        if is_island(o_name, islands):
            o = island(o_name, _rows_k(dense_t(pre + "self_attn.", ("o_proj",)), model.rank, sh.hq_local * cfg.head_dim))
        else:
            o_q, o_s = model._shard_rows(*r.linear(pre + "self_attn.o_proj"), sh.hq_local * cfg.head_dim)
            o = Int4Linear(o_name, o_q.to(dev).contiguous(), o_s.to(dev).contiguous())
        if is_island(gu_name, islands):
            wt = dense_t(pre + "mlp.", ("gate_proj", "up_proj"))
            gate_up = island(gu_name, model._shard_gate_up(wt, wt[:1])[0])
        else:
            gu = [r.linear(pre + "mlp.%s_proj" % p) for p in ("gate", "up")]
            gu_q, gu_s = model._shard_gate_up(torch.cat([a for a, _ in gu], 1), torch.cat([b for _, b in gu], 1))
            gate_up = Int4Linear(gu_name, gu_q.to(dev).contiguous(), gu_s.to(dev).contiguous())
        if is_island(dn_name, islands):
            down = island(dn_name, _rows_k(dense_t(pre + "mlp.", ("down_proj",)), model.rank, sh.inter_local))
        else:
            dn_q, dn_s = model._shard_rows(*r.linear(pre + "mlp.down_proj"), sh.inter_local)
            down = Int4Linear(dn_name, dn_q.to(dev).contiguous(), dn_s.to(dev).contiguous())
        return LayerWeights(
            input_norm=r.get(pre + "input_layernorm.weight").to(dev, torch.bfloat16),
            post_norm=r.get(pre + "post_attention_layernorm.weight").to(dev, torch.bfloat16),
            qkv=qkv, o=o, gate_up=gate_up, down=down)

    n_layers = len(model.layers) or cfg.num_layers
    model.layers = [layer("model.layers.%d." % i, "model.layers.%d." % i) for i in range(n_layers)]
    if model.mtp is not None or (r.has("mtp.eh_proj.qweight") and mc.mtp_layers):
        if r.has("mtp.eh_proj.qweight"):
            eq, es = r.linear("mtp.eh_proj")
            model.mtp = MTPWeights(
                enorm=r.get("mtp.enorm.weight").to(dev, torch.bfloat16),
                hnorm=r.get("mtp.hnorm.weight").to(dev, torch.bfloat16),
                norm=r.get("mtp.norm.weight").to(dev, torch.bfloat16),
                eh_proj=Int4Linear("mtp.eh_proj", eq.to(dev), es.to(dev)),
                layer=layer("mtp.layers.0.", "mtp.layers.0."))
    model.final_norm = r.get("model.norm.weight").to(dev, torch.bfloat16)
    v0, v1 = model.vocab_start, model.vocab_start + sh.vocab_local
    from safetensors import safe_open
    with open(os.path.join(path, "config.json")) as f:
        side = json.load(f).get("embed_tokens_quant", {})
    with safe_open(os.path.join(path, side.get("side_file", SIDE_FILE)), framework="pt") as h:
        codes = h.get_slice(side.get("key_weight", "embed_tokens.int8"))[v0:v1]
        scales = h.get_slice(side.get("key_scale", "embed_tokens.scale"))[v0:v1]
    model.embed_codes = codes.to(dev).contiguous()
    model.embed_scales = scales.reshape(-1).to(dev, torch.float16).contiguous()
    model.lm_head = Int8RowLinear("lm_head", r.get("lm_head.weight")[v0:v1].to(dev).contiguous(),
                                  r.get("lm_head.weight_scale")[v0:v1].reshape(-1).to(dev, torch.float16))
    if model.rope is None:
        model.rope = rope_table(mc.max_position, mc.head_dim, mc.rope_theta, dev)
