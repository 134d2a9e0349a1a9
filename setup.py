"""Build the scirs_b200 CUDA extension in-tree for sm_100a (B200).

    python setup.py build_ext --inplace

Every kernel is compiled for `-gencode arch=compute_100a,code=sm_100a` only.
"""
import glob
import os

from setuptools import setup
from torch.utils.cpp_extension import BuildExtension, CppExtension, CUDAExtension

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join("scirs_b200", "csrc")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + [
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "--expt-relaxed-constexpr",
    "-DNDEBUG",
    "-U__CUDA_NO_HALF_OPERATORS__",
    "-U__CUDA_NO_BFLOAT16_CONVERSIONS__",
    "-U__CUDA_NO_HALF_CONVERSIONS__",
    "-U__CUDA_NO_BFLOAT162_OPERATORS__",
]
if os.environ.get("SCIRS_KCHECK") == "1":  # debug build: internal index checks -> status word
    NVCC_FLAGS.append("-DSCIRS_KCHECK")
if os.environ.get("SCIRS_PTXAS_VERBOSE"):
    NVCC_FLAGS.append("-Xptxas=-v")
CXX_FLAGS = ["-O3", "-std=c++17"]


def _sources(names):
    return [os.path.join(CSRC, n) for n in names]


ext_modules = [
    CUDAExtension(
        name="scirs_b200._C",
        sources=_sources(
            [
                "bindings.cpp",
                "host_common.cpp",
                "gemm_sm100.cu",
                "norm_loss.cu",
                "optim.cu",
                "attention.cu",
                "attention_sm100.cu",
                "vision.cu",
                "tp.cu",
                "attention_fwd_sm100.cu",
                "attention_bwd_sm100.cu",
                "paged_attention.cu",
                "conv.cu",
                "elementwise.cu",
                "rnn.cu",
            ]
        ),
        extra_compile_args={"cxx": CXX_FLAGS, "nvcc": NVCC_FLAGS},
    ),
    CppExtension(
        name="scirs_b200._data",
        sources=_sources(["dataloader.cpp", "host_runtime.cpp"]),
        extra_compile_args={"cxx": CXX_FLAGS},
    ),
    CUDAExtension(
        name="scirs_b200._comm",
        sources=_sources(["comm_bindings.cpp", "host_common.cpp", "comm.cu"]),
        extra_compile_args={"cxx": CXX_FLAGS, "nvcc": NVCC_FLAGS},
    ),
]

class _BuildExt(BuildExtension):
    """One build directory per extension, so each keeps its own ninja log and
    dependency state (incremental rebuilds recompile only what changed)."""

    def build_extension(self, ext):
        old = self.build_temp
        self.build_temp = os.path.join(old, ext.name.rsplit(".", 1)[-1])
        try:
            super().build_extension(ext)
        finally:
            self.build_temp = old


setup(
    name="scirs_b200",
    version="0.1.0",
    packages=["scirs_b200"],
    package_data={"scirs_b200": ["configs/*.yaml"]},
    ext_modules=ext_modules,
    cmdclass={"build_ext": _BuildExt.with_options(use_ninja=True)},
)
