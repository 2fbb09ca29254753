"""Hash of the native sources, embedded in the kernel library at build time.

``setup.py`` compiles ``source_hash(csrc)`` into the library and the loader
compares it with the tree next to the package, so a library built from other
sources (a stale in-tree build that travelled with a snapshot, or sources
edited since) is refused instead of being run. The reference namespaces its
compile caches by configuration for the same reason, so that stale
artefacts cannot bypass a changed hook (``k8v4_v030/launch.sh:29,161``).
"""
from __future__ import annotations

import hashlib
import os

SUFFIXES = (".cu", ".cuh", ".cpp", ".h", ".hpp")


def source_files(csrc: str) -> list[str]:
    out = []
    for dirpath, _, names in os.walk(csrc):
        out += [os.path.join(dirpath, n) for n in names if n.endswith(SUFFIXES)]
    return sorted(out, key=lambda p: os.path.relpath(p, csrc))


def source_hash(csrc: str) -> str:
    """16 hex digits of SHA-256 over every source's relative path and bytes."""
    h = hashlib.sha256()
    for p in source_files(csrc):
        h.update(os.path.relpath(p, csrc).replace(os.sep, "/").encode())
        h.update(b"\0")
        with open(p, "rb") as f:
            h.update(f.read())
        h.update(b"\0")
    return h.hexdigest()[:16]
