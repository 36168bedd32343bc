"""Build the sm_100a extension in place: ``python setup.py build_ext --inplace``.

Every CUDA source is compiled for ``compute_100a``/``sm_100a`` only (passed
explicitly, so torch's own arch list is bypassed) with ``-lineinfo``.
"""
import glob
import os

from setuptools import setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension

ROOT = os.path.dirname(os.path.abspath(__file__))
CUDA_FLAGS = ["-O3", "-gencode", "arch=compute_100a,code=sm_100a", "-lineinfo", "-std=c++17",
              "--expt-relaxed-constexpr"]
if os.environ.get("RT_PTXAS_VERBOSE"):
    CUDA_FLAGS += ["-Xptxas", "-v"]


def sources():
    cu = sorted(glob.glob(os.path.join("csrc", "**", "*.cu"), recursive=True))
    return ["csrc/bindings.cpp"] + cu


setup(
    name="rwkv_theseus_b200",
    version="0.1.0",
    packages=["rwkv_theseus_b200", "rwkv_theseus_b200.models", "rwkv_theseus_b200.ops",
              "rwkv_theseus_b200.parallel", "rwkv_theseus_b200.convert"],
    ext_modules=[CUDAExtension(
        name="rwkv_theseus_b200._C",
        sources=sources(),
        include_dirs=[os.path.join(ROOT, "csrc")],
        extra_compile_args={"cxx": ["-O3", "-std=c++17"], "nvcc": CUDA_FLAGS},
    )],
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
)
