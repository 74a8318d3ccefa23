"""Build the dion_b200 CUDA extension in-tree for sm_100a.

    python setup.py build_ext --inplace

produces dion_b200/_C.*.so (the sm_100a kernels) and dion_b200/_io.*.so
(host-side data loading, plain C++) next to the Python sources.
"""
import glob
import os

from setuptools import setup
from torch.utils.cpp_extension import BuildExtension, CppExtension, CUDAExtension

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join("dion_b200", "csrc")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + [
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "--expt-relaxed-constexpr",
    "-U__CUDA_NO_HALF_OPERATORS__",
    "-U__CUDA_NO_HALF_CONVERSIONS__",
    "-U__CUDA_NO_BFLOAT16_CONVERSIONS__",
    "-U__CUDA_NO_BFLOAT162_OPERATORS__",
]
if os.environ.get("BDION_PTXAS_VERBOSE"):
    NVCC_FLAGS.append("-Xptxas=-v")

# Link the shared C++ runtime that torch itself loads. A toolchain whose
# libstdc++.so development link is missing silently embeds the static archive
# instead, and torch's error checks (which format their messages with
# iostreams) then crash inside the extension rather than raising.
LINK_CXX_RUNTIME = ["-l:libstdc++.so.6"]

sources = sorted(glob.glob(os.path.join(CSRC, "*.cu"))) + sorted(glob.glob(os.path.join(CSRC, "*.cpp")))

setup(
    name="dion_b200",
    ext_modules=[
        CUDAExtension(
            name="dion_b200._C",
            sources=sources,
            include_dirs=[os.path.join(HERE, CSRC)],
            extra_compile_args={"cxx": ["-O3", "-std=c++17"], "nvcc": NVCC_FLAGS},
            extra_link_args=LINK_CXX_RUNTIME,
        ),
        CppExtension(
            name="dion_b200._io",
            sources=[os.path.join(CSRC, "io", "token_loader.cpp")],
            extra_compile_args=["-O3", "-std=c++17", "-pthread"],
            extra_link_args=["-pthread"] + LINK_CXX_RUNTIME,
        ),
    ],
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
)
