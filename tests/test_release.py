"""AutoRound -> GPTQ adaptation and release staging (CPU), on a checkpoint the
bake tool writes."""
import json
import os

import pytest
import torch
from safetensors import safe_open
from safetensors.torch import save_file

from k8v4_xpu_b200.models.checkpoint import load_checkpoint
from k8v4_xpu_b200.models.config import TINY
from k8v4_xpu_b200.models.dense import DenseModel
from k8v4_xpu_b200.tools import bake, release


def _autoround_copy(tmp_path, drop_g_idx=True):
    """A random GPTQ checkpoint relabelled as AutoRound's auto_gptq packing,
    without g_idx tensors (AutoRound does not write them)."""
    ck = tmp_path / "ar"
    bake.random_checkpoint(str(ck), "tiny", layers=2, mtp=False)
    cfg = json.loads((ck / "config.json").read_text())
    cfg["quantization_config"] = {"packing_format": "auto_round:auto_gptq", "bits": 4, "group_size": 128,
                                  "sym": True, "quant_method": "auto-round"}
    (ck / "config.json").write_text(json.dumps(cfg))
    if drop_g_idx:
        for f in ck.glob("*.safetensors"):
            with safe_open(str(f), "pt") as h:
                t = {k: h.get_tensor(k) for k in h.keys() if not k.endswith(".g_idx")}
            save_file(t, str(f))
        idx = ck / "model.safetensors.index.json"
        if idx.exists():
            doc = json.loads(idx.read_text())
            doc["weight_map"] = {k: v for k, v in doc["weight_map"].items() if not k.endswith(".g_idx")}
            idx.write_text(json.dumps(doc))
    return ck


def _tensors(ck):
    out = {}
    for f in ck.glob("*.safetensors"):
        with safe_open(str(f), "pt") as h:
            out.update({k: h.get_tensor(k) for k in h.keys()})
    return out


def test_adapt_autoround_adds_group_indices_and_keeps_weights(tmp_path):
    ck = _autoround_copy(tmp_path)
    before = _tensors(ck)
    rec = release.adapt_autoround(ck, expect_linears=2 * 7)  # q, k, v, o, gate, up, down per layer
    assert rec["linears_verified"] == 14 and rec["added_group_indices"] == 14 and not rec["changed_weight_values"]
    after = _tensors(ck)
    for k, v in before.items():
        assert torch.equal(after[k], v), k  # no payload rewritten
    gi = [k for k in after if k.endswith(".g_idx")]
    assert len(gi) == 14
    qkv = "model.layers.0.self_attn.q_proj"
    K = before[qkv + ".qweight"].shape[0] * 8
    assert torch.equal(after[qkv + ".g_idx"], torch.arange(K, dtype=torch.int32) // 128)
    cfg = json.loads((ck / "config.json").read_text())
    assert cfg["quantization_config"]["quant_method"] == "gptq" and cfg["quantization_config"]["desc_act"] is False
    assert (ck / "config.json.upstream").exists() and (ck / "COMPATIBILITY.json").exists()
    # the adapted checkpoint still loads into the model
    m = DenseModel(TINY.__class__(**{**TINY.__dict__, "num_layers": 2}), device="cpu")
    load_checkpoint(m, str(ck))
    with pytest.raises(RuntimeError):
        release.adapt_autoround(ck)  # a second run is refused


def test_adapt_autoround_refuses_asymmetric_zeros_and_other_formats(tmp_path):
    ck = _autoround_copy(tmp_path)
    def has_zeros(f):
        with safe_open(str(f), "pt") as h:
            return any(k.endswith(".qzeros") for k in h.keys())
    f = next(f for f in sorted(ck.glob("*.safetensors")) if has_zeros(f))
    with safe_open(str(f), "pt") as h:
        t = {k: h.get_tensor(k) for k in h.keys()}
    zk = next(k for k in t if k.endswith(".qzeros"))
    t[zk] = t[zk].clone()
    t[zk].view(-1)[0] = 0x77777778  # one nibble 8: not the symmetric zero point
    save_file(t, str(f))
    with pytest.raises(ValueError, match="symmetric zero point"):
        release.adapt_autoround(ck)
    cfg = json.loads((ck / "config.json").read_text())
    cfg["quantization_config"]["sym"] = False
    (ck / "config.json").write_text(json.dumps(cfg))
    with pytest.raises(ValueError, match="symmetric"):
        release.adapt_autoround(ck)


def test_stage_release_annotates_changed_shards_and_links_the_rest(tmp_path):
    ck = tmp_path / "ck"
    bake.random_checkpoint(str(ck), "tiny", layers=1, mtp=False)
    shards = sorted(p.name for p in ck.glob("*.safetensors"))
    changed = shards[-1]
    dst = tmp_path / "pub"
    man = release.stage_release(ck, dst, "modified for test", changed=(changed,), source_repo="org/base")
    h, _ = release.read_header(dst / changed)
    assert h["__metadata__"]["modification_notice"] == "modified for test"
    assert _tensors(dst) == {} or all(torch.equal(v, _tensors(ck)[k]) for k, v in _tensors(dst).items())
    for s in shards:
        if s != changed:
            assert os.stat(dst / s).st_ino == os.stat(ck / s).st_ino  # hard link, not a copy
    mods = json.loads((dst / "MODIFICATIONS.json").read_text())
    assert changed in mods["files"] and len(mods["files"][changed]["tensor_payload_sha256"]) == 64
    cfg = json.loads((dst / "config.json").read_text())
    assert cfg["_derivative_of"] == "org/base" and cfg["_modification_notice"] == "modified for test"
    assert man["indexed_tensors"] > 0 and "RELEASE_FILES.json" not in man["files"]
    with pytest.raises(ValueError):
        release.stage_release(ck, dst, "again")
