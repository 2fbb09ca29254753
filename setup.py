"""Build the k8v4 sm_100a kernel library in-tree: k8v4_xpu_b200/_C*.so.

    python setup.py build_ext --inplace

Every CUDA source is compiled for sm_100a only (tcgen05 / TMA / TMEM code).
"""
import glob
import os

from setuptools import setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension

ROOT = os.path.dirname(os.path.abspath(__file__))


def _source_hash() -> str:
    # the package module, loaded by path (importing the package needs torch's extension first)
    import importlib.util
    spec = importlib.util.spec_from_file_location("_k8v4_buildhash", os.path.join(ROOT, "k8v4_xpu_b200", "buildhash.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod.source_hash(os.path.join(ROOT, "csrc"))


SOURCE_HASH = ['-DK8V4_SOURCE_HASH="%s"' % _source_hash()]
SOURCES = ["csrc/bindings.cpp"] + sorted(glob.glob("csrc/**/*.cu", recursive=True))
NVCC = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "--expt-relaxed-constexpr",
    "-diag-suppress", "20044",
] + os.environ.get("K8V4_NVCC_EXTRA", "").split()

setup(
    name="k8v4_xpu_b200",
    version="0.1.0",
    packages=[],
    ext_modules=[
        CUDAExtension(
            name="k8v4_xpu_b200._C",
            sources=SOURCES,
            include_dirs=[os.path.join(ROOT, "csrc")],
            extra_compile_args={"cxx": ["-O3", "-std=c++17"] + SOURCE_HASH, "nvcc": NVCC},
        )
    ],
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
    entry_points={
        "vllm.general_plugins": ["k8v4_int8_k_int4_v = k8v4_xpu_b200.registry:register_vllm"],
        "console_scripts": ["k8v4-serve = k8v4_xpu_b200.cli:main", "k8v4-bake = k8v4_xpu_b200.tools.bake:main"],
    },
)
