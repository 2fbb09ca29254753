"""Cache dtype registry and the vLLM registration (CPU; vLLM files are copied, never edited)."""
import os
import shutil

import pytest
import torch

from k8v4_xpu_b200 import registry


def test_own_registry():
    assert registry.kv_cache_torch_dtype("int8_k_int4_v") == torch.uint8
    with pytest.raises(ValueError):
        registry.kv_cache_torch_dtype("fp8")


def test_patch_vllm_tree_on_a_copy(tmp_path):
    vllm = pytest.importorskip("vllm")
    root = os.path.dirname(vllm.__file__)
    for rel in ("config/cache.py", "utils/torch_utils.py"):
        dst = tmp_path / rel
        dst.parent.mkdir(parents=True, exist_ok=True)
        shutil.copy(os.path.join(root, rel), dst)
    r = registry.patch_vllm_tree(str(tmp_path))
    assert r == {"config/cache.py": "patched", "utils/torch_utils.py": "patched"}
    assert registry.patch_vllm_tree(str(tmp_path)) == {"config/cache.py": "already",
                                                       "utils/torch_utils.py": "already"}
    src = (tmp_path / "config/cache.py").read_text()
    lit = src[src.index("CacheDType = Literal["):]
    assert '"int8_k_int4_v"' in lit[:lit.index("]")]
    compile(src, "cache.py", "exec")
    compile((tmp_path / "utils/torch_utils.py").read_text(), "torch_utils.py", "exec")
    # the installed package itself is untouched
    assert '"int8_k_int4_v"' not in open(os.path.join(root, "config/cache.py")).read()


def test_patch_refuses_unknown_layout(tmp_path):
    (tmp_path / "config").mkdir()
    (tmp_path / "utils").mkdir()
    (tmp_path / "config/cache.py").write_text("x = 1\n")
    (tmp_path / "utils/torch_utils.py").write_text("y = 2\n")
    with pytest.raises(RuntimeError):
        registry.patch_vllm_tree(str(tmp_path))


def test_register_vllm_runtime():
    pytest.importorskip("vllm")
    assert registry.register_vllm()
    from vllm.utils import torch_utils
    from vllm.v1.attention.backends.registry import _ATTN_OVERRIDES, AttentionBackendEnum
    assert torch_utils.STR_DTYPE_TO_TORCH_DTYPE["int8_k_int4_v"] == torch.uint8
    assert _ATTN_OVERRIDES[AttentionBackendEnum.CUSTOM] == registry.BACKEND_PATH
