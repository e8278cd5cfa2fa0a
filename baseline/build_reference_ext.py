"""Build the reference's own attention extension (unmodified ``csrc/ext.cpp`` + ``csrc/flash_attn_sm75.cu``) for
sm_100 into the installed reference tree ``baseline/_ref/flashattention_custom/``.

The reference's ``setup.py`` only adds the extension when ``torch.cuda.is_available()``, which is false on a build
host without a GPU, so ``pip install`` produced a pure-Python install whose ops fall back to per-head Python loops.
This script compiles the same sources with the same flags as the reference's ``setup.py`` (``-O3 --use_fast_math
-lineinfo -std=c++17`` and the half-operator undefines) and the arch list ``TORCH_CUDA_ARCH_LIST=10.0`` that the
baseline plan names, so the reference arm runs its stock CUDA kernels.

Usage: python baseline/build_reference_ext.py [--src /path/to/reference]
"""
import argparse
import os
import shutil
import sys
import tempfile

HERE = os.path.dirname(os.path.abspath(__file__))
REF = os.path.join(HERE, "_ref")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--src", default=os.environ.get("HRM_REFERENCE_SRC", ""),
                    help="reference source tree (or set HRM_REFERENCE_SRC)")
    args = ap.parse_args()
    if not args.src:
        ap.error("give the reference source tree with --src or HRM_REFERENCE_SRC")
    os.environ["TORCH_CUDA_ARCH_LIST"] = "10.0"
    from torch.utils.cpp_extension import load
    tmp = tempfile.mkdtemp(prefix="refext_")
    srcs = []
    for f in ("ext.cpp", "flash_attn_sm75.cu"):
        d = os.path.join(tmp, f)
        shutil.copy(os.path.join(args.src, "csrc", f), d)
        srcs.append(d)
    build_dir = os.path.join(tmp, "build")
    os.makedirs(build_dir)
    load(name="_ext", sources=srcs, build_directory=build_dir, verbose=False,
         extra_cflags=["-O3", "-std=c++17"],
         extra_cuda_cflags=["-O3", "--use_fast_math", "-lineinfo", "-std=c++17",
                            "-U__CUDA_NO_HALF_OPERATORS__", "-U__CUDA_NO_HALF_CONVERSIONS__",
                            "-U__CUDA_NO_HALF2_OPERATORS__",
                            "-gencode", "arch=compute_100,code=sm_100"],
         is_python_module=True)
    so = [f for f in os.listdir(build_dir) if f.endswith(".so")]
    if not so:
        sys.exit("build produced no .so")
    dst = os.path.join(REF, "flashattention_custom", "_ext.so")
    shutil.copy(os.path.join(build_dir, so[0]), dst)
    print("built", dst)


if __name__ == "__main__":
    main()
