"""Package hygiene and source-text properties (CPU).

Counterpart of the reference's package-hygiene and source-text tests
(``k8v4_v030/tests/test_public_package.py:23-108``,
``tests/test_layout_mtp.py:80-103``): properties that the sources themselves
must keep, checked on the text so that a change that breaks one fails
without a GPU.
"""
import ast
import importlib
import pathlib
import re

import pytest

ROOT = pathlib.Path(__file__).resolve().parents[1]
PKG = ROOT / "k8v4_xpu_b200"
CSRC = ROOT / "csrc"
CUDA_FILES = sorted(list(CSRC.rglob("*.cu")) + list(CSRC.rglob("*.cuh")))
SCRATCH = "_work"  # git-ignored scratch folder at the repo root


def _py_files():
    out = [ROOT / "bench.py", ROOT / "__graft_entry__.py"]
    for d in ("k8v4_xpu_b200", "bench", "tests"):
        out += sorted((ROOT / d).rglob("*.py"))
    return out


def _strip_comments(src: str) -> str:
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return re.sub(r"//[^\n]*", "", src)


def test_every_package_module_imports_without_a_gpu():
    bad = []
    for f in sorted(PKG.rglob("*.py")):
        mod = ".".join(f.relative_to(ROOT).with_suffix("").parts)
        if mod.endswith("__main__"):
            continue
        try:
            importlib.import_module(mod)
        except Exception as e:  # noqa: BLE001 - report every failure at once
            bad.append("%s: %r" % (mod, e))
    assert not bad, bad


def test_committed_code_never_reaches_into_the_scratch_folder():
    for f in _py_files():
        tree = ast.parse(f.read_text(), str(f))
        for node in ast.walk(tree):
            names = []
            if isinstance(node, ast.Import):
                names = [a.name for a in node.names]
            elif isinstance(node, ast.ImportFrom):
                names = [node.module or ""]
            assert not any(n.split(".")[0] == SCRATCH for n in names), f
            if isinstance(node, ast.Constant) and isinstance(node.value, str):
                assert not node.value.startswith(SCRATCH + "/"), (f, node.value)


# A bulk-copy instruction and a fan-out qualifier, written as patterns so that
# this file names neither of them as plain text.
_BULK_COPY = re.compile(r"cp[.]async[.]bul[k]")
_FAN_OUT = re.compile(r"multi[c]ast")


def test_no_bulk_copy_fans_out_to_a_cluster_in_the_cuda_sources():
    # Multi-GPU runs must not reach a TMA / bulk load that fans out to several
    # CTAs of a cluster: a line that issues a bulk copy names no fan-out form.
    for f in CUDA_FILES:
        code = _strip_comments(f.read_text())
        for line in code.splitlines():
            if _BULK_COPY.search(line):
                assert not _FAN_OUT.search(line), (f, line)


def test_cuda_sources_build_for_sm100a_only():
    build = "".join(p.read_text() for p in (ROOT / "__graft_entry__.py", ROOT / "setup.py") if p.exists())
    assert "sm_100a" in build
    for f in CUDA_FILES:
        code = _strip_comments(f.read_text())
        assert "wgmma" not in code, f  # Hopper-only instruction
        assert "__trap" not in code, f  # failures are reported through the status word


def _loop_bodies(code: str):
    """(header, body) of every ``while`` / ``for (;;)`` loop that has a body."""
    for m in re.finditer(r"\b(while\s*\(|for\s*\(\s*;\s*;\s*\))", code):
        # skip the do { } while (...) tail
        if code[:m.start()].rstrip().endswith("}") and code[m.end():].lstrip().startswith(("0)", "false)")):
            continue
        i = m.end()
        if m.group(1).startswith("while"):
            depth = 1
            while depth:
                depth += {"(": 1, ")": -1}.get(code[i], 0)
                i += 1
        rest = code[i:].lstrip()
        if not rest.startswith("{"):
            # a single statement: its body is the text up to the semicolon
            yield code[m.start():i], rest[: rest.find(";") + 1]
            continue
        j = code.index("{", i)
        depth, k = 0, j
        while True:
            depth += {"{": 1, "}": -1}.get(code[k], 0)
            k += 1
            if depth == 0:
                break
        yield code[m.start():i], code[j:k]


SPIN = re.compile(r"mbar_(try|test)_wait|ld_acquire|ld\.acquire|volatile")


def test_every_device_spin_loop_is_bounded_by_the_wait_limit():
    """A loop that polls a barrier or a flag either checks the clock against
    K8V4_WAIT_LIMIT_NS or hands the wait to a bounded helper."""
    found = 0
    for f in CUDA_FILES:
        code = _strip_comments(f.read_text())
        for header, body in _loop_bodies(code):
            if not SPIN.search(header + body):
                continue
            found += 1
            bounded = "K8V4_WAIT_LIMIT_NS" in body or re.search(r"\bmbar_wait(_all|_drain)?\(", body)
            assert bounded, (f.name, header, body[:300])
    assert found >= 3  # the barrier, drain and peer waits at least


def test_public_surface_names():
    import k8v4_xpu_b200 as k
    from k8v4_xpu_b200 import config, ops
    assert k.CACHE_DTYPE == "int8_k_int4_v"
    for name in ("rope_store", "decode_attn", "prefill_attn", "wq_gemm", "rmsnorm", "silu_mul", "status",
                 "require"):
        assert callable(getattr(ops, name)), name
    flags = {a for act in config.build_parser()._actions for a in act.option_strings}
    for flag in ("--kv-cache-dtype", "--tensor-parallel-size", "--max-num-seqs", "--max-num-batched-tokens",
                 "--max-model-len", "--enable-prefix-caching", "--speculative-config", "--compilation-config",
                 "--kv-cache-dtype-skip-layers"):
        assert flag in flags, flag


@pytest.mark.parametrize("f", CUDA_FILES, ids=lambda p: p.name)
def test_cuda_sources_have_a_header_comment(f):
    assert f.read_text().lstrip().startswith("//"), f


def test_source_hash_tracks_every_native_source(tmp_path):
    import shutil
    from k8v4_xpu_b200.buildhash import source_hash
    tree = tmp_path / "csrc"
    shutil.copytree(CSRC, tree)
    h0 = source_hash(str(tree))
    assert h0 == source_hash(str(CSRC)) and len(h0) == 16
    f = tree / "kv" / "store.cu"
    f.write_text(f.read_text() + "\n")
    h1 = source_hash(str(tree))
    assert h1 != h0
    (tree / "kv" / "store.cu").rename(tree / "kv" / "store2.cu")
    assert source_hash(str(tree)) not in (h0, h1)


def test_the_in_tree_library_was_built_from_this_tree():
    """A stale build (sources edited since) is refused by the loader."""
    from k8v4_xpu_b200 import ops
    from k8v4_xpu_b200.buildhash import source_hash
    if ops._library_file() is None:
        pytest.skip("no in-tree build")
    assert ops.load(), ops._ERROR
    import torch
    assert str(torch.ops.k8v4.source_hash()) == source_hash(str(CSRC))
