"""Build the sm_100a kernels in-tree.

    python setup.py build_ext --inplace

produces ``parallel_b200/_C*.so``.  Only ``sm_100a`` code is generated
(tcgen05 / TMA / TMEM instructions exist on no other target), and torch's own
arch list is bypassed by passing the gencode flags explicitly.
"""
import glob
import os

from setuptools import find_packages, setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension

ROOT = os.path.dirname(os.path.abspath(__file__))
os.environ.setdefault("TORCH_CUDA_ARCH_LIST", "10.0a")

NVCC_FLAGS = [
    "-O3",
    "-std=c++17",
    "-gencode",
    "arch=compute_100a,code=sm_100a",
    "-lineinfo",
    "--expt-relaxed-constexpr",
    "-Xptxas=-v" if os.environ.get("PB_PTXAS_VERBOSE") else "-Xptxas=-O3",
    "-DNDEBUG",
]
CXX_FLAGS = ["-O3", "-std=c++17"]


def sources():
    srcs = sorted(glob.glob(os.path.join("csrc", "*.cu")) + glob.glob(os.path.join("csrc", "*.cpp")))
    return [os.path.relpath(s, ROOT) if os.path.isabs(s) else s for s in srcs]


setup(
    name="parallel_b200",
    version="0.1.0",
    packages=find_packages(include=["parallel_b200", "parallel_b200.*"]),
    package_data={"parallel_b200": ["conf/*.yaml"]},
    ext_modules=[
        CUDAExtension(
            name="parallel_b200._C",
            sources=sources(),
            include_dirs=[os.path.join(ROOT, "csrc")],
            extra_compile_args={"cxx": CXX_FLAGS, "nvcc": NVCC_FLAGS},
        )
    ],
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
    entry_points={"console_scripts": ["parallel-b200-train = parallel_b200.train:main"]},
)
