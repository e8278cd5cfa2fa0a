"""Build of hrm_flashrenderer_b200 and its sm_100a CUDA extension (in-tree: ``python setup.py build_ext --inplace``).

The extension is compiled for ``sm_100a`` only (tcgen05 / TMEM / TMA); torch's own arch list is bypassed by
passing ``-gencode`` directly.  The HRM retrieval core (C++17) is built separately by ``hrm_core/Makefile``.
"""
import os
from setuptools import setup, find_packages

ROOT = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(ROOT, "csrc")

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "--expt-relaxed-constexpr",
    "-U__CUDA_NO_HALF_OPERATORS__", "-U__CUDA_NO_HALF_CONVERSIONS__",
    "-U__CUDA_NO_BFLOAT16_CONVERSIONS__", "-U__CUDA_NO_HALF2_OPERATORS__",
]
CXX_FLAGS = ["-O3", "-std=c++17"]

CUDA_SOURCES = ["bindings.cpp", "gemm_w8a16.cu", "gemm_chain.cu", "norm.cu", "attention.cu", "attention_tc.cu", "comm.cu",
                "gemm_noalloc.cu", "gemm_nt.cu", "flash_train.cu", "sampling.cu", "pho.cu",
                "train_ops.cu"]


def ext_modules():
    from torch.utils.cpp_extension import CUDAExtension
    return [CUDAExtension(
        name="hrm_flashrenderer_b200._C",
        sources=[os.path.join("csrc", s) for s in CUDA_SOURCES],
        include_dirs=[CSRC],
        extra_compile_args={"cxx": CXX_FLAGS, "nvcc": NVCC_FLAGS},
    )]


def cmdclass():
    from torch.utils.cpp_extension import BuildExtension
    return {"build_ext": BuildExtension.with_options(use_ninja=True)}


setup(
    name="hrm_flashrenderer_b200",
    version="0.1.0",
    description="B200-native retrieval-augmented tensor-parallel LLM inference (HRM FlashRenderer capabilities)",
    packages=find_packages(exclude=("tests", "tests.*", "_work", "_work.*")),
    ext_modules=ext_modules(),
    cmdclass=cmdclass(),
    entry_points={
        "console_scripts": [
            "hrm-flash=hrm_flashrenderer_b200.serving.cli:main",
            "hrm-flashd=hrm_flashrenderer_b200.serving.daemon:main",
            "hrm-flash-serve=hrm_flashrenderer_b200.serving.serve:main",
            "hrm-flash-router=hrm_flashrenderer_b200.serving.router:main",
            "flash-kernel-test=hrm_flashrenderer_b200.compat.kernel_test:kernel_test_main",
            "flash-append-test=hrm_flashrenderer_b200.compat.kernel_test:append_test_main",
        ]
    },
)
