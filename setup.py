"""Build the native runtime in-tree: ``python setup.py build_ext --inplace``.

Produces ``weightbridge_b200/_C*.so`` (sm_100a kernels, CPU executor, IPC/VMM/multicast).
"""
import os

from setuptools import find_packages, setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join("weightbridge_b200", "csrc")

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo", "-O3", "-std=c++17",
    "--expt-relaxed-constexpr",
]

setup(
    name="weightbridge_b200",
    version="0.1.0",
    packages=find_packages(include=["weightbridge_b200", "weightbridge_b200.*", "wbridge"]),
    ext_modules=[
        CUDAExtension(
            name="weightbridge_b200._C",
            sources=[os.path.join(CSRC, f) for f in
                     ("wb_bindings.cpp", "wb_transfer.cu", "wb_splitq.cu", "wb_noalloc.cu", "wb_synth.cu", "wb_board.cpp", "wb_ipc.cpp",
                      "wb_cpu.cpp")],
            include_dirs=[os.path.join(HERE, CSRC)],
            extra_compile_args={"cxx": ["-O3", "-std=c++17"], "nvcc": NVCC_FLAGS},
        )
    ],
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
)
