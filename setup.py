"""Build of the package's native extension for B200 (sm_100a only).

    python setup.py build_ext --inplace

compiles every ``vllm_cmp170hx_b200/csrc/*.cu`` / ``*.cpp`` into
``vllm_cmp170hx_b200/_C*.so`` (in the source tree, so it is importable from a
checkout and travels with it).  The architecture flag is given explicitly,
which also keeps torch from adding its own arch list.
"""

import glob
import os

from setuptools import setup

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = "vllm_cmp170hx_b200"
CSRC = os.path.join(PKG, "csrc")

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH_FLAGS + [
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "--expt-relaxed-constexpr",
    "-DNDEBUG",
    "-U__CUDA_NO_HALF_OPERATORS__",
    "-U__CUDA_NO_HALF_CONVERSIONS__",
    "-U__CUDA_NO_BFLOAT16_CONVERSIONS__",
    "-U__CUDA_NO_HALF2_OPERATORS__",
]
CXX_FLAGS = ["-O3", "-std=c++17"]


def _sources():
    cu = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    cpp = sorted(glob.glob(os.path.join(CSRC, "*.cpp")))
    return cu + cpp


def ext_modules():
    from torch.utils.cpp_extension import CUDAExtension

    return [
        CUDAExtension(
            name=f"{PKG}._C",
            sources=_sources(),
            include_dirs=[os.path.join(ROOT, CSRC)],
            extra_compile_args={"cxx": CXX_FLAGS, "nvcc": NVCC_FLAGS},
        )
    ]


if __name__ == "__main__":
    from torch.utils.cpp_extension import BuildExtension

    os.environ.setdefault("MAX_JOBS", str(os.cpu_count() or 8))
    setup(
        name=PKG,
        version="0.1.0",
        packages=[PKG],
        ext_modules=ext_modules(),
        cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
    )
