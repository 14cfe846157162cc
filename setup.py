"""Builds the sm_100a extension in-tree: `python setup.py build_ext --inplace`.

Only sm_100a (B200) code is generated: the arch flags below bypass PyTorch's own
arch list.
"""
import glob
import os

from setuptools import setup

os.environ.setdefault("TORCH_CUDA_ARCH_LIST", "10.0a")
from torch.utils.cpp_extension import BuildExtension, CUDAExtension  # noqa: E402

HERE = os.path.dirname(os.path.abspath(__file__))
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + [
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "--expt-relaxed-constexpr",
    "--expt-extended-lambda",
    "-Xptxas=-v" if os.environ.get("DMAD_PTXAS_VERBOSE") else "-Xptxas=-O3",
    "-U__CUDA_NO_HALF_OPERATORS__",
    "-U__CUDA_NO_BFLOAT16_CONVERSIONS__",
    "-U__CUDA_NO_BFLOAT16_OPERATORS__",
]
if os.environ.get("DMAD_BOUNDS_CHECK"):
    NVCC_FLAGS.append("-DDMAD_BOUNDS_CHECK=1")

sources = sorted(glob.glob(os.path.join("csrc", "*.cu"))) + sorted(glob.glob(os.path.join("csrc", "*.cpp")))

setup(
    name="dmad_b200",
    version="0.1.0",
    packages=["dmad_b200"],
    ext_modules=[
        CUDAExtension(
            name="dmad_b200._C",
            sources=sources,
            include_dirs=[os.path.join(HERE, "csrc")],
            extra_compile_args={"cxx": ["-O3", "-std=c++17"], "nvcc": NVCC_FLAGS},
        )
    ],
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
)
