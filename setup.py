"""Build script for the minisgl native library (sm_100a only).

    python setup.py build_ext --inplace      # development: _C*.so next to the sources
    pip install --no-build-isolation .      # installable package (metadata in pyproject.toml)

The in-place build produces ``minisgl/_C*.so`` next to the Python sources,
so the built library travels with a copy of the source tree.
"""

import os

from setuptools import setup

NVCC_FLAGS = [
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "-gencode=arch=compute_100a,code=sm_100a",
    "--expt-relaxed-constexpr",
    "-Xptxas=-v" if os.environ.get("MINISGL_PTXAS_VERBOSE") else "-Xptxas=-O3",
    "-DNDEBUG",
]
CXX_FLAGS = ["-O3", "-std=c++17", "-DNDEBUG"]

SOURCES = [
    "minisgl/csrc/binding.cpp",
    "minisgl/csrc/radix.cpp",
    "minisgl/csrc/gemm.cu",
    "minisgl/csrc/gemm_persistent.cu",
    "minisgl/csrc/gemm_streamk.cu",
    "minisgl/csrc/attention.cu",
    "minisgl/csrc/elementwise.cu",
    "minisgl/csrc/rope_store.cu",
    "minisgl/csrc/sampling.cu",
    "minisgl/csrc/moe.cu",
    "minisgl/csrc/symm.cu",
    "minisgl/csrc/mla.cu",
    "minisgl/csrc/mxfp4.cu",
    "minisgl/csrc/mx_gemm.cu",
    "minisgl/csrc/ep.cu",
]


def ext_modules():
    from torch.utils.cpp_extension import CUDAExtension

    return [
        CUDAExtension(
            name="minisgl._C",
            sources=SOURCES,
            extra_compile_args={"cxx": CXX_FLAGS, "nvcc": NVCC_FLAGS},
        )
    ]


def cmdclass():
    from torch.utils.cpp_extension import BuildExtension

    return {"build_ext": BuildExtension.with_options(use_ninja=True)}


if __name__ == "__main__":
    # torch's own arch list must not add other targets: the gencode above is the only one
    os.environ["TORCH_CUDA_ARCH_LIST"] = "10.0a"
    from setuptools import find_packages

    setup(
        packages=find_packages(include=["minisgl", "minisgl.*"]),
        ext_modules=ext_modules(),
        cmdclass=cmdclass(),
    )
