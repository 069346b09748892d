"""Builds the sm_100a CUDA extension in place: ``python setup.py build_ext --inplace``.

Every .cu file is compiled for ``-gencode arch=compute_100a,code=sm_100a`` only; the
extension is written into ``drivedit_b200/`` so it travels with the source tree.
"""
import glob
import os

from setuptools import setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension

ROOT = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(ROOT, "csrc")

sources = sorted(
    glob.glob(os.path.join(CSRC, "**", "*.cu"), recursive=True)
    + glob.glob(os.path.join(CSRC, "**", "*.cpp"), recursive=True)
)
# host-only C++ data runtime is a separate extension
sources = [s for s in sources if os.sep + "data" + os.sep not in s]

nvcc_flags = [
    "-O3",
    "-std=c++17",
    "-gencode=arch=compute_100a,code=sm_100a",
    "-lineinfo",
    "--use_fast_math",
    "--expt-relaxed-constexpr",
    "-Xptxas=-v" if os.environ.get("DDB_PTXAS_VERBOSE") else "-Xptxas=-O3",
    "-DNDEBUG",
]

data_sources = sorted(glob.glob(os.path.join(CSRC, "data", "*.cpp")))
ext_modules = [
        CUDAExtension(
            name="drivedit_b200._C",
            sources=[os.path.relpath(s, ROOT) for s in sources],
            include_dirs=[CSRC],
            extra_compile_args={"cxx": ["-O3", "-std=c++17"], "nvcc": nvcc_flags},
        ),
]
if data_sources:
    from torch.utils.cpp_extension import CppExtension

    ext_modules.append(
        CppExtension(
            name="drivedit_b200._data",
            sources=[os.path.relpath(s, ROOT) for s in data_sources],
            include_dirs=[CSRC],
            extra_compile_args=["-O3", "-std=c++17", "-pthread"],
            libraries=["z"],
            extra_link_args=["-pthread"],
        )
    )

setup(
    name="drivedit_b200_ext",
    ext_modules=ext_modules,
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
)
