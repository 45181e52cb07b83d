"""Build of bitscom_b200: one in-tree CUDA extension, ``bitscom_b200._C``.

    python setup.py build_ext --inplace      # what __graft_entry__.build() runs
    pip install --no-build-isolation -e .    # editable install

Every .cu file is compiled for sm_100a only (``-gencode
arch=compute_100a,code=sm_100a``); passing the explicit -gencode keeps
torch.utils.cpp_extension from adding its own architecture list.  The
reference's setup.py (setup.py:222-238) passed no architecture at all.
"""

import os

from setuptools import find_packages, setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension

ROOT = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(ROOT, "csrc")

SOURCES = [
    "csrc/bindings.cpp",
    "csrc/runtime/comm.cpp",
    "csrc/backend/process_group_lowbit.cpp",
    "csrc/kernels/quant_kernels.cu",
    "csrc/kernels/lowbit_coll.cu",
    "csrc/kernels/noalloc_allreduce.cu",
]

NVCC_FLAGS = [
    "-gencode=arch=compute_100a,code=sm_100a",
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "--expt-relaxed-constexpr",
    "-Xptxas=-v" if os.environ.get("BITSCOM_PTXAS_VERBOSE") else "-Xptxas=-O3",
]
CXX_FLAGS = ["-O3", "-std=c++17", "-DUSE_C10D_NCCL"]

setup(
    name="bitscom_b200",
    version="0.1.0",
    description="Blackwell-native low-bit gradient communication for PyTorch",
    packages=find_packages(include=["bitscom_b200", "bitscom_b200.*"]),
    package_data={"bitscom_b200.tuning": ["*.json"]},
    ext_modules=[
        CUDAExtension(
            name="bitscom_b200._C",
            sources=SOURCES,
            include_dirs=[CSRC],
            extra_compile_args={"cxx": CXX_FLAGS, "nvcc": NVCC_FLAGS},
            # Link the C++ runtime dynamically: a toolchain that silently
            # falls back to libstdc++.a would give this module a private copy
            # of the library (bound locally by -Bsymbolic-functions) that then
            # mixes with the process's libstdc++ (e.g. its locale facets) and
            # crashes on the first formatted integer.
            extra_link_args=["-l:libstdc++.so.6"],
            libraries=["cuda"],
        )
    ],
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
    python_requires=">=3.10",
)
