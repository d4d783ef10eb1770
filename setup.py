"""Build the native extension in place:

    python setup.py build_ext --inplace

Produces ``ring_attention_benchmark_b200/_C*.so`` containing every sm_100a
kernel and the native ring runtime.  The CUDA code is compiled for sm_100a only
(``-gencode arch=compute_100a,code=sm_100a``); torch's own arch list is bypassed
because an explicit ``-gencode`` flag is passed.
"""
import glob
import os

from setuptools import setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension

ROOT = os.path.dirname(os.path.abspath(__file__))


def _nccl_paths():
    import nvidia.nccl  # shipped with the torch wheel

    base = os.path.dirname(nvidia.nccl.__file__) if nvidia.nccl.__file__ else list(
        nvidia.nccl.__path__)[0]
    return os.path.join(base, "include"), os.path.join(base, "lib")


NCCL_INC, NCCL_LIB = _nccl_paths()

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + [
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "--expt-relaxed-constexpr",
    "-DNDEBUG",
    "-Xptxas=-warn-spills",
]
if os.environ.get("RAB_PTXAS_VERBOSE"):
    NVCC_FLAGS.append("-Xptxas=-v")
# RAB_DEBUG_BOUNDS=1: index checks in the flash kernels that report through the
# device status word instead of faulting (see csrc/include/status.h)
if os.environ.get("RAB_DEBUG_BOUNDS") == "1":
    NVCC_FLAGS.append("-DRAB_DEBUG_BOUNDS")
CXX_FLAGS = ["-O3", "-std=c++17", "-DNDEBUG"]

sources = sorted(
    glob.glob(os.path.join("csrc", "*.cpp"))
    + glob.glob(os.path.join("csrc", "runtime", "*.cpp"))
    + glob.glob(os.path.join("csrc", "kernels", "*.cu"))
)

setup(
    name="ring_attention_benchmark_b200",
    version="0.1.0",
    packages=[
        "ring_attention_benchmark_b200",
        "ring_attention_benchmark_b200.models",
        "ring_attention_benchmark_b200.ops",
        "ring_attention_benchmark_b200.parallel",
        "ring_attention_benchmark_b200.utils",
    ],
    ext_modules=[
        CUDAExtension(
            name="ring_attention_benchmark_b200._C",
            sources=sources,
            include_dirs=[os.path.join(ROOT, "csrc", "include"), NCCL_INC],
            library_dirs=[NCCL_LIB],
            libraries=[":libnccl.so.2", "rt"],
            extra_link_args=[f"-Wl,-rpath,{NCCL_LIB}"],
            extra_compile_args={"cxx": CXX_FLAGS, "nvcc": NVCC_FLAGS},
        )
    ],
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
)
