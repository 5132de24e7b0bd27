"""Build the squish_b200 native extension in-tree for sm_100a.

    python setup.py build_ext --inplace

produces squish_b200/_C*.so (CUDA kernels for sm_100a + the C++ CPU reference library).
"""
import glob
import os

from setuptools import find_packages, setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join("squish_b200", "csrc")

cuda_sources = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
cpp_sources = [os.path.join(CSRC, "bindings.cpp"), os.path.join(CSRC, "cpu_ref.cpp"), os.path.join(CSRC, "entropy.cpp"),
               os.path.join(CSRC, "host_utils.cpp"), os.path.join(CSRC, "grammar.cpp"),
               os.path.join(CSRC, "quant_research.cpp"), os.path.join(CSRC, "kv_research.cpp"),
               os.path.join(CSRC, "recurrent.cpp")]

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "--expt-relaxed-constexpr",
    "-Xptxas", "-warn-spills",
]
if os.environ.get("SQ_PTXAS_VERBOSE"):
    NVCC_FLAGS += ["-Xptxas", "-v"]

setup(
    name="squish_b200",
    version="0.1.0",
    packages=find_packages(include=["squish_b200", "squish_b200.*"]),
    package_data={"squish_b200.serving": ["static/*.html"]},
    entry_points={"console_scripts": ["squish=squish_b200.cli:main"]},
    ext_modules=[
        CUDAExtension(
            name="squish_b200._C",
            sources=cpp_sources + cuda_sources,
            extra_compile_args={
                "cxx": ["-O3", "-std=c++17"],
                "nvcc": NVCC_FLAGS,
            },
        )
    ],
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
)
