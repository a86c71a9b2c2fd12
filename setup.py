"""Build the native sm_100a extension in-tree:  python setup.py build_ext --inplace

Every .cu/.cpp under mamformer_b200/csrc is compiled for sm_100a only
(-gencode arch=compute_100a,code=sm_100a); the resulting mamformer_b200/_C*.so is loaded by
mamformer_b200.ops.  A second module, mamformer_b200._C_check, holds a bounds-checked build of
the index-driven kernels (MAMF_BOUNDS_CHECK: bad indices are recorded and skipped, never
accessed); MAMF_BOUNDS_CHECK=1 in the environment builds the main module with the checks too.
"""

import glob
import os

from setuptools import setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join("mamformer_b200", "csrc")

NVCC_FLAGS = [
    "-O3", "-lineinfo", "-std=c++17",
    "-gencode", "arch=compute_100a,code=sm_100a",
    "--expt-relaxed-constexpr", "--expt-extended-lambda",
    "-U__CUDA_NO_HALF_OPERATORS__", "-U__CUDA_NO_HALF_CONVERSIONS__",
    "-U__CUDA_NO_BFLOAT16_CONVERSIONS__", "-U__CUDA_NO_BFLOAT16_OPERATORS__",
    "-DNDEBUG",
]
if os.environ.get("MAMF_BOUNDS_CHECK") == "1":
    NVCC_FLAGS.append("-DMAMF_BOUNDS_CHECK=1")

sources = sorted(glob.glob(os.path.join(CSRC, "*.cu")) + glob.glob(os.path.join(CSRC, "*.cpp")))
# Bounds-checked build of the index-driven kernels (always built; see csrc/check/).
# The wrappers under csrc/check/ include the kernel files with MAMF_BOUNDS_CHECK defined, so their
# objects never collide with the main module's.
CHECK_SOURCES = sorted(glob.glob(os.path.join(CSRC, "check", "*.cu")) + glob.glob(os.path.join(CSRC, "check", "*.cpp")))
CHECK_FLAGS = [f for f in NVCC_FLAGS if f != "-DMAMF_BOUNDS_CHECK=1"]

setup(
    name="mamformer_b200",
    version="0.1.0",
    packages=["mamformer_b200"],
    ext_modules=[
        CUDAExtension(
            name="mamformer_b200._C",
            sources=sources,
            include_dirs=[os.path.join(HERE, CSRC)],
            extra_compile_args={"cxx": ["-O3", "-std=c++17"], "nvcc": NVCC_FLAGS},
        ),
        CUDAExtension(
            name="mamformer_b200._C_check",
            sources=CHECK_SOURCES,
            include_dirs=[os.path.join(HERE, CSRC)],
            extra_compile_args={"cxx": ["-O3", "-std=c++17"], "nvcc": CHECK_FLAGS},
        ),
    ],
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
)
