"""Build the sm_100a extension in place:  ``python setup.py build_ext --inplace``.

Only Blackwell (sm_100a) code is generated; nvcc cross-compiles it on a host
without a GPU.  ``MAX_JOBS`` controls ninja parallelism.
"""

from __future__ import annotations

import glob
import os

from setuptools import setup

from torch.utils.cpp_extension import BuildExtension, CUDAExtension

ROOT = os.path.dirname(os.path.abspath(__file__))

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH_FLAGS + [
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "--expt-relaxed-constexpr",
    "-U__CUDA_NO_HALF_OPERATORS__",
    "-U__CUDA_NO_HALF_CONVERSIONS__",
    "-U__CUDA_NO_BFLOAT16_OPERATORS__",
    "-U__CUDA_NO_BFLOAT16_CONVERSIONS__",
    "-U__CUDA_NO_HALF2_OPERATORS__",
]
if os.environ.get("LRB_PTXAS_VERBOSE"):
    NVCC_FLAGS.append("-Xptxas=-v")


def sources(*patterns: str) -> list[str]:
    out: list[str] = []
    for pat in patterns:
        out.extend(sorted(glob.glob(os.path.join(ROOT, pat))))
    return [os.path.relpath(p, ROOT) for p in out]


def extensions():
    return [
        CUDAExtension(
            name="llm_research_b200._C",
            sources=sources("csrc/bindings.cpp", "csrc/kernels/*.cu", "csrc/comm/*.cu"),
            include_dirs=[os.path.join(ROOT, "csrc")],
            extra_compile_args={"cxx": ["-O3", "-std=c++17"], "nvcc": NVCC_FLAGS},
        ),
    ]


if __name__ == "__main__":
    # torch appends -gencode flags derived from TORCH_CUDA_ARCH_LIST; pin it to
    # the one target so no other architecture is built.
    os.environ["TORCH_CUDA_ARCH_LIST"] = "10.0a"
    setup(
        name="llm_research_b200",
        version="0.1.0",
        packages=[],
        ext_modules=extensions(),
        cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
    )
