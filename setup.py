"""Build the sm_100a CUDA extension of sparsecache_b200 in place.

    python setup.py build_ext --inplace

The kernels are written for Blackwell (sm_100a) only: tcgen05/TMEM tensor-core
instructions and TMA tiled loads do not exist on other architectures, so the
arch flags are passed explicitly instead of using torch's arch list.
"""
import os
from pathlib import Path

from setuptools import find_packages, setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension

ROOT = Path(__file__).resolve().parent
CSRC = ROOT / "sparsecache_b200" / "ops" / "csrc"

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "--expt-relaxed-constexpr",
    "-Xptxas", "-v" if os.environ.get("SC_PTXAS_VERBOSE") else "-O3",
]

ext = CUDAExtension(
    name="sparsecache_b200.ops._C",
    sources=[str(p.relative_to(ROOT)) for p in sorted(CSRC.glob("*.cu"))]
    + [str(p.relative_to(ROOT)) for p in sorted(CSRC.glob("*.cpp"))],
    include_dirs=[str(CSRC)],
    extra_compile_args={"cxx": ["-O3", "-std=c++17"], "nvcc": NVCC_FLAGS},
)

setup(
    name="sparsecache_b200",
    version="0.1.0",
    packages=find_packages(include=["sparsecache_b200", "sparsecache_b200.*"]),
    ext_modules=[ext],
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
    entry_points={
        "console_scripts": [
            "sparsecache-prepare=sparsecache_b200.data:main",
            "sparsecache-precompute=sparsecache_b200.precompute:main",
            "sparsecache-qa=sparsecache_b200.qa:main",
            "sparsecache-train=sparsecache_b200.training.cli:main",
            "sparsecache-eval=sparsecache_b200.evaluation.cli:main",
            "sparsecache-feasibility=sparsecache_b200.pipelines.feasibility:main",
            "sparsecache-pd=sparsecache_b200.pipelines.pd:main",
        ]
    },
)
