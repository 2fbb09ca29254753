"""Registration of the ``int8_k_int4_v`` cache dtype and the K8/V4 attention backend.

The reference makes stock vLLM accept its cache dtype by splicing text into
the installed source (``k8v4_v030/patch_installed_vllm.py:16-149``): the
dtype list of ``config/cache.py``, the dtype -> storage map of
``utils/torch_utils.py`` and the platform's backend selector. Here:

* ``CACHE_DTYPES`` / ``kv_cache_torch_dtype``: this framework's own registry
  (the engine and the backend look the dtype up here);
* ``register_vllm()``: a ``vllm.general_plugins`` entry point. It registers
  :class:`~k8v4_xpu_b200.attention.backend.K8V4AttentionBackend` as vLLM's
  ``CUSTOM`` attention backend and maps the dtype to ``torch.uint8`` in the
  running process (vLLM's runtime registration API, no file edits);
* ``patch_vllm_tree(root)``: the remaining piece vLLM cannot take at run
  time, the dtype's entry in the ``CacheDType`` literal (validated by
  pydantic), spliced idempotently into a vLLM source tree the caller points
  at (an image build, a copy); it never edits anything on its own.

Serving through vLLM itself is outside this framework's tests: the built-in
engine serves; the backend class follows vLLM's V1 method names.
"""
from __future__ import annotations

import os
import re

import torch

from .kv.layout import CACHE_DTYPE

CACHE_DTYPES: dict[str, torch.dtype] = {CACHE_DTYPE: torch.uint8}
BACKEND_PATH = "k8v4_xpu_b200.attention.backend.K8V4AttentionBackend"


def kv_cache_torch_dtype(name: str) -> torch.dtype:
    if name not in CACHE_DTYPES:
        raise ValueError("unknown kv_cache_dtype %r (registered: %s)" % (name, sorted(CACHE_DTYPES)))
    return CACHE_DTYPES[name]


def register_vllm() -> bool:
    """vLLM plugin entry point. Returns False when vLLM is not importable."""
    try:
        from vllm.utils import torch_utils
        from vllm.v1.attention.backends.registry import AttentionBackendEnum, register_backend
    except Exception:
        return False
    torch_utils.STR_DTYPE_TO_TORCH_DTYPE.setdefault(CACHE_DTYPE, torch.uint8)
    register_backend(AttentionBackendEnum.CUSTOM, BACKEND_PATH)
    return True


_LITERAL = re.compile(r"(CacheDType\s*=\s*Literal\[\s*\n)")
_DTYPE_MAP = re.compile(r"(STR_DTYPE_TO_TORCH_DTYPE\s*=\s*\{\s*\n)")


def patch_vllm_tree(root: str) -> dict[str, str]:
    """Splice the dtype into ``config/cache.py`` and ``utils/torch_utils.py``
    under ``root`` (a vLLM package directory). Idempotent; returns
    {file: "patched" | "already" }; raises if an anchor is missing."""
    results = {}
    for rel, rx, line in (("config/cache.py", _LITERAL, '    "%s",\n' % CACHE_DTYPE),
                          ("utils/torch_utils.py", _DTYPE_MAP, '    "%s": torch.uint8,\n' % CACHE_DTYPE)):
        path = os.path.join(root, rel)
        with open(path) as f:
            src = f.read()
        if '"%s"' % CACHE_DTYPE in src:
            results[rel] = "already"
            continue
        m = rx.search(src)
        if m is None:
            raise RuntimeError("anchor not found in %s (vLLM layout changed)" % path)
        src = src[:m.end()] + line + src[m.end():]
        with open(path, "w") as f:
            f.write(src)
        results[rel] = "patched"
    return results
