"""Build the astrai_b200 CUDA extension in-tree for B200 (sm_100a only).

    python setup.py build_ext --inplace -j 16

produces astrai_b200/_C.*.so. Only sm_100a SASS is generated: the kernels use
tcgen05 / TMEM / TMA instructions that exist on no other architecture.
"""
import glob
import os

os.environ.setdefault("TORCH_CUDA_ARCH_LIST", "10.0a")

from setuptools import find_packages, setup  # noqa: E402
from torch.utils.cpp_extension import BuildExtension, CUDAExtension  # noqa: E402

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join("astrai_b200", "csrc")
sources = sorted(glob.glob(os.path.join(CSRC, "*.cu")) + glob.glob(os.path.join(CSRC, "*.cpp")))

NVCC_FLAGS = [
    "-gencode=arch=compute_100a,code=sm_100a",
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "--expt-relaxed-constexpr",
    "-Xptxas=-warn-spills",
    "-DNDEBUG",
]

# name, version and dependencies live in pyproject.toml
setup(
    packages=find_packages(include=["astrai_b200*", "astrai"]),
    ext_modules=[
        CUDAExtension(
            name="astrai_b200._C",
            sources=sources,
            include_dirs=[os.path.join(HERE, CSRC)],
            extra_compile_args={"cxx": ["-O3", "-std=c++17"], "nvcc": NVCC_FLAGS},
        )
    ],
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
)
