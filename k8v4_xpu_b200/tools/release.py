"""Checkpoint publication tools (the reference's T7 / T8).

``adapt_autoround``
    Makes an AutoRound checkpoint packed as ``auto_round:auto_gptq`` (int4,
    group 128, symmetric) loadable as plain GPTQ, as the reference's
    ``tools/prepare_swift_autoround.py`` does: every ``.qweight`` is checked
    (int32 ``[K/8, N]``, K a multiple of 128) together with its ``qzeros``
    (every packed nibble 7, i.e. the symmetric zero point 8), a missing
    ``g_idx`` (``k // 128``) is added in a separate shard, the upstream
    config and index are kept beside the new ones (``*.upstream``), the
    quantization config becomes ``gptq`` with ``desc_act`` off and the dense
    modules listed as exclusions, and ``COMPATIBILITY.json`` records what
    changed. No weight payload is rewritten; a second run is refused.

``stage_release``
    A publication copy of a checkpoint (``tools/prepare_swift_hf_release.py``):
    unchanged shards are hard links, the shards listed as changed get a
    modification notice in their safetensors header metadata while their
    tensor bytes are copied unchanged (their SHA-256 is recorded), JSON
    metadata files carry the notice, and ``MODIFICATIONS.json`` plus
    ``RELEASE_FILES.json`` (every file and its size) are written. Every tensor
    of the index must be found in its shard's header.

A safetensors file is an 8-byte little-endian header length, a JSON header
(tensor name -> dtype, shape, payload byte range; optional ``__metadata__``
of strings) padded to 8 bytes, then the payload.

    python -m k8v4_xpu_b200.tools.release adapt CHECKPOINT [--linears N]
    python -m k8v4_xpu_b200.tools.release stage --src DIR --dst NEW --notice TEXT [--changed SHARD ...]
"""
from __future__ import annotations

import argparse
import hashlib
import json
import os
import shutil
import struct
from pathlib import Path

GROUP = 128
SYM_ZERO_WORD = 0x77777777  # eight nibbles of 7: GPTQ stores zero point 8 as 8 - 1
# modules that stay dense in the served checkpoint (the MTP head and any vision
# tower); a GPTQ loader skips them
DENSE_EXCLUSIONS = {"-:.*visual.*": {}, "-:.*mtp.*": {}}


# ------------------------------------------------------------- safetensors io
def read_header(path: Path) -> tuple[dict, int]:
    """``(header, payload_start)`` of one safetensors file."""
    with open(path, "rb") as f:
        (n,) = struct.unpack("<Q", f.read(8))
        return json.loads(f.read(n)), 8 + n


def _encode_header(header: dict) -> bytes:
    raw = json.dumps(header, separators=(",", ":")).encode()
    return raw + b" " * ((-len(raw)) % 8)


def _tensor_bytes(path: Path, header: dict, start: int, name: str) -> bytes:
    lo, hi = header[name]["data_offsets"]
    with open(path, "rb") as f:
        f.seek(start + lo)
        return f.read(hi - lo)


def _weight_map(ckpt: Path) -> tuple[dict[str, str], dict | None]:
    """tensor -> shard file name, and the index document when there is one."""
    idx_path = ckpt / "model.safetensors.index.json"
    if idx_path.exists():
        idx = json.loads(idx_path.read_text())
        return dict(idx["weight_map"]), idx
    shards = sorted(p.name for p in ckpt.glob("*.safetensors"))
    wm = {}
    for s in shards:
        h, _ = read_header(ckpt / s)
        wm.update({k: s for k in h if k != "__metadata__"})
    return wm, None


# ------------------------------------------------------------ AutoRound -> GPTQ
def adapt_autoround(ckpt: str | Path, expect_linears: int | None = None) -> dict:
    """Adapt an AutoRound (auto_gptq packing) checkpoint in place for a GPTQ
    loader; returns the compatibility record."""
    p = Path(ckpt).resolve()
    if (p / "COMPATIBILITY.json").exists():
        raise RuntimeError("%s was adapted already; start again from an upstream copy" % p)
    cfg = json.loads((p / "config.json").read_text())
    q = cfg.get("quantization_config") or {}
    want = {"packing_format": "auto_round:auto_gptq", "bits": 4, "group_size": GROUP, "sym": True}
    bad = {k: q.get(k) for k, v in want.items() if q.get(k) != v}
    if bad:
        raise ValueError("not an int4 / group-128 / symmetric auto_gptq-packed checkpoint: %s" % bad)
    wm, idx = _weight_map(p)
    headers: dict[str, tuple[dict, int]] = {}

    def hdr(shard: str):
        if Path(shard).name != shard:
            raise ValueError("shard %r is not a plain file name" % shard)
        if shard not in headers:
            headers[shard] = read_header(p / shard)
        return headers[shard]

    added: dict[str, list[int]] = {}
    linears = 0
    for key in sorted(wm):
        if not key.endswith(".qweight"):
            continue
        base = key[: -len(".qweight")]
        h, _ = hdr(wm[key])
        info = h[key]
        if info["dtype"] != "I32" or len(info["shape"]) != 2:
            raise ValueError("%s: qweight must be a 2D int32 tensor, got %s %s" % (base, info["dtype"], info["shape"]))
        k = info["shape"][0] * 8
        if k % GROUP:
            raise ValueError("%s: K = %d is not a whole number of %d-wide groups" % (base, k, GROUP))
        zkey = base + ".qzeros"
        if zkey not in wm:
            raise ValueError("%s: no qzeros" % base)
        zh, zstart = hdr(wm[zkey])
        zeros = _tensor_bytes(p / wm[zkey], zh, zstart, zkey)
        if any(w != SYM_ZERO_WORD for (w,) in struct.iter_unpack("<I", zeros)):
            raise ValueError("%s: qzeros are not the symmetric zero point (every nibble 7)" % base)
        if base + ".g_idx" not in wm:
            added[base + ".g_idx"] = [i // GROUP for i in range(k)]
        linears += 1
    if expect_linears is not None and linears != expect_linears:
        raise ValueError("found %d GPTQ linears, expected %d" % (linears, expect_linears))

    new_shard = "compat_g_idx.safetensors"
    if added:
        header, blobs, at = {}, [], 0
        for name, vals in added.items():
            raw = struct.pack("<%di" % len(vals), *vals)
            header[name] = {"dtype": "I32", "shape": [len(vals)], "data_offsets": [at, at + len(raw)]}
            blobs.append(raw)
            at += len(raw)
        tmp = p / (new_shard + ".partial")
        with open(tmp, "wb") as f:
            enc = _encode_header(header)
            f.write(struct.pack("<Q", len(enc)) + enc)
            for b in blobs:
                f.write(b)
        os.replace(tmp, p / new_shard)
    # keep the upstream metadata beside the adapted files
    for name in ("config.json", "model.safetensors.index.json"):
        if (p / name).exists():
            shutil.copy2(p / name, p / (name + ".upstream"))
    gptq = {"quant_method": "gptq", "bits": 4, "group_size": GROUP, "sym": True, "desc_act": False,
            "lm_head": False, "dynamic": dict(DENSE_EXCLUSIONS)}
    cfg["quantization_config"] = gptq
    (p / "config.json").write_text(json.dumps(cfg, indent=2) + "\n")
    (p / "quantize_config.json").write_text(json.dumps(gptq, indent=2) + "\n")
    if added:
        if idx is None:  # a single-file checkpoint gains an index naming both shards
            idx = {"metadata": {}, "weight_map": dict(wm)}
        idx["weight_map"].update({n: new_shard for n in added})
        meta = idx.setdefault("metadata", {})
        meta["total_size"] = int(meta.get("total_size", 0)) + sum(4 * len(v) for v in added.values())
        (p / "model.safetensors.index.json").write_text(json.dumps(idx, indent=2) + "\n")
    record = {"source_format": q["packing_format"], "linears_verified": linears,
              "zero_points": "every packed nibble 7 (GPTQ zero point 8)", "added_group_indices": len(added),
              "changed_weight_values": False}
    (p / "COMPATIBILITY.json").write_text(json.dumps(record, indent=2) + "\n")
    return record


# ----------------------------------------------------------- release staging
def _annotate_shard(src: Path, dst: Path, notice: str) -> str:
    """Copy a shard with ``notice`` in its header metadata; the payload bytes
    are streamed unchanged and their SHA-256 returned."""
    header, start = read_header(src)
    header.setdefault("__metadata__", {})["modification_notice"] = notice
    enc = _encode_header(header)
    digest = hashlib.sha256()
    with open(src, "rb") as r, open(dst, "xb") as w:
        w.write(struct.pack("<Q", len(enc)) + enc)
        r.seek(start)
        while True:
            block = r.read(8 << 20)
            if not block:
                break
            digest.update(block)
            w.write(block)
    return digest.hexdigest()


def _payload_sha256(path: Path) -> str:
    _, start = read_header(path)
    digest = hashlib.sha256()
    with open(path, "rb") as f:
        f.seek(start)
        while True:
            block = f.read(8 << 20)
            if not block:
                break
            digest.update(block)
    return digest.hexdigest()


def stage_release(src: str | Path, dst: str | Path, notice: str, changed: tuple[str, ...] = (),
                  source_repo: str | None = None) -> dict:
    """Stage a publication copy of checkpoint ``src`` in the new directory ``dst``."""
    src, dst = Path(src).resolve(), Path(dst).resolve()
    if dst.exists() or dst == src:
        raise ValueError("the destination must be a new directory, separate from the source")
    dst.mkdir(parents=True)
    mods: dict[str, dict] = {}
    for f in sorted(src.iterdir()):
        if not f.is_file() or f.name.endswith((".upstream", ".partial")):
            continue
        out = dst / f.name
        if f.suffix == ".safetensors":
            if f.name in changed:
                sha = _annotate_shard(f, out, notice)
                if sha != _payload_sha256(f):
                    raise RuntimeError("payload of %s changed while staging" % f.name)
                mods[f.name] = {"notice": notice, "tensor_payload_sha256": sha}
            else:
                os.link(f, out)  # same bytes, no copy
        elif f.suffix == ".json":
            doc = json.loads(f.read_text())
            if isinstance(doc, dict):
                doc["_modification_notice"] = notice
                if f.name == "config.json" and source_repo:
                    doc["_derivative_of"] = source_repo
                mods[f.name] = {"notice": notice}
            out.write_text(json.dumps(doc, indent=2) + "\n")
        else:
            shutil.copyfile(f, out)
    # every indexed tensor must be present in the header of its shard
    wm, _ = _weight_map(dst)
    seen: dict[str, dict] = {}
    for tensor, shard in wm.items():
        if shard not in seen:
            seen[shard] = read_header(dst / shard)[0]
        if tensor not in seen[shard]:
            raise RuntimeError("%s is indexed in %s but missing from its header" % (tensor, shard))
    (dst / "MODIFICATIONS.json").write_text(json.dumps({"source": source_repo, "files": mods}, indent=2) + "\n")
    files = {str(f.relative_to(dst)): f.stat().st_size for f in sorted(dst.rglob("*")) if f.is_file()}
    manifest = {"files": files, "total_bytes": sum(files.values()), "indexed_tensors": len(wm)}
    (dst / "RELEASE_FILES.json").write_text(json.dumps(manifest, indent=2) + "\n")
    return manifest


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="k8v4-release")
    sub = ap.add_subparsers(dest="cmd", required=True)
    a = sub.add_parser("adapt", help="AutoRound (auto_gptq packing) -> GPTQ loader config, in place")
    a.add_argument("checkpoint")
    a.add_argument("--linears", type=int, help="expected number of GPTQ linears")
    s = sub.add_parser("stage", help="stage a publication copy")
    s.add_argument("--src", required=True)
    s.add_argument("--dst", required=True)
    s.add_argument("--notice", required=True)
    s.add_argument("--changed", nargs="*", default=[], help="shards whose headers get the notice")
    s.add_argument("--source-repo")
    args = ap.parse_args(argv)
    if args.cmd == "adapt":
        print(json.dumps(adapt_autoround(args.checkpoint, args.linears)))
    else:
        print(json.dumps(stage_release(args.src, args.dst, args.notice, tuple(args.changed), args.source_repo)))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
