"""Build script for vllm_musa_b200.

The native extension ``vllm_musa_b200._C`` holds every sm_100a CUDA kernel (csrc/**/*.cu,
compiled for ``arch=compute_100a,code=sm_100a`` only) plus the C++ host runtime
(csrc/runtime).  Build in place so the shared object sits inside the package tree:

    python setup.py build_ext --inplace
"""
import glob
import os

from setuptools import find_packages, setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension

ROOT = os.path.dirname(os.path.abspath(__file__))

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "--expt-relaxed-constexpr",
    "-Xptxas=-warn-spills",
    "-DNDEBUG",
]
CXX_FLAGS = ["-O3", "-std=c++17", "-DNDEBUG"]


def _sources():
    cu = sorted(glob.glob(os.path.join("csrc", "**", "*.cu"), recursive=True))
    cpp = sorted(glob.glob(os.path.join("csrc", "**", "*.cpp"), recursive=True))
    return cu + cpp


setup(
    name="vllm_musa_b200",
    version="0.1.0",
    description="Blackwell-native (sm_100a) LLM serving framework with vllm-musa's capabilities",
    packages=find_packages(include=["vllm_musa_b200", "vllm_musa_b200.*"]),
    package_data={"vllm_musa_b200": ["tuning/*.json"]},
    ext_modules=[
        CUDAExtension(
            name="vllm_musa_b200._C",
            sources=_sources(),
            include_dirs=[os.path.join(ROOT, "csrc")],
            extra_compile_args={"cxx": CXX_FLAGS, "nvcc": NVCC_FLAGS},
        )
    ],
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
    entry_points={
        "vllm.platform_plugins": ["b200 = vllm_musa_b200:b200_platform_plugin"],
        "vllm.general_plugins": ["b200_custom_ops = vllm_musa_b200:register_custom_ops"],
        "console_scripts": [
            "b200-vllm = vllm_musa_b200.entrypoints.cli:main",
            "b200_collect_env = vllm_musa_b200.collect_env:main",
        ],
    },
    python_requires=">=3.10",
)
