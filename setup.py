"""Build the native parts of test1_b200 in-tree.

    python setup.py build_ext --inplace

Two extensions:
  * test1_b200._host  -- C++ host runtime: LayerAdam SIMD kernels (AVX-512 /
    AVX2 / scalar chosen at run time), worker pool, shared-memory regions and
    counters, CPU slot reduce, NUMA placement.
  * test1_b200._cuda  -- sm_100a CUDA kernels (tcgen05 GEMM, attention,
    RMSNorm, RoPE, SwiGLU, cross-entropy, embedding, fused collectives),
    compiled only for `-gencode arch=compute_100a,code=sm_100a`.
  * test1_b200._cuda_checked -- with T1_BUILD_CHECKED=1 only: the same
    kernels built with -DT1_BOUNDS_CHECK (every instrumented index is
    range-checked; the first out-of-bounds access per kernel file is recorded
    and skipped, read back with `bounds_errors()`).  Selected at run time by
    T1_BOUNDS_CHECK=1.
"""
import glob
import os

from setuptools import setup
from torch.utils.cpp_extension import BuildExtension, CppExtension, CUDAExtension

ROOT = os.path.dirname(os.path.abspath(__file__))
HOST_DIR = os.path.join("test1_b200", "csrc", "host")
CUDA_DIR = os.path.join("test1_b200", "csrc", "cuda")


def host_extension():
    sources = sorted(glob.glob(os.path.join(HOST_DIR, "*.cpp")))
    return CppExtension(
        name="test1_b200._host",
        sources=sources,
        extra_compile_args={"cxx": ["-O3", "-std=c++17", "-fno-math-errno", "-Wno-unused-function"]},
    )


def _checked_sources(sources):
    """One wrapper per source under build/ that includes it, so the checked
    objects never share paths (or ninja rules) with the normal ones."""
    out_dir = os.path.join("build", "checked_src")
    os.makedirs(out_dir, exist_ok=True)
    out = []
    for src in sources:
        dst = os.path.join(out_dir, os.path.basename(src))
        text = f'#include "{os.path.join(ROOT, src)}"\n'
        if not os.path.exists(dst) or open(dst).read() != text:
            with open(dst, "w") as f:
                f.write(text)
        out.append(dst)
    return out


def cuda_extension(checked=False):
    sources = sorted(glob.glob(os.path.join(CUDA_DIR, "*.cu"))) + sorted(
        glob.glob(os.path.join(CUDA_DIR, "*.cpp"))
    )
    if not sources:
        return None
    defines = ["-DT1_BOUNDS_CHECK"] if checked else []
    if checked:
        sources = _checked_sources(sources)
    nvcc_flags = [
        "-O3",
        "-std=c++17",
        "-gencode",
        "arch=compute_100a,code=sm_100a",
        "-lineinfo",
        "--expt-relaxed-constexpr",
        "-U__CUDA_NO_HALF_OPERATORS__",
        "-U__CUDA_NO_HALF_CONVERSIONS__",
        "-U__CUDA_NO_BFLOAT16_CONVERSIONS__",
        "-U__CUDA_NO_BFLOAT16_OPERATORS__",
        "-Xptxas=-v" if os.environ.get("T1_PTXAS_VERBOSE") else "-Xptxas=-O3",
    ]
    return CUDAExtension(
        name="test1_b200._cuda_checked" if checked else "test1_b200._cuda",
        sources=sources,
        include_dirs=[os.path.join(ROOT, CUDA_DIR)],
        extra_compile_args={"cxx": ["-O3", "-std=c++17"] + defines, "nvcc": nvcc_flags + defines},
    )


exts = [host_extension()]
if os.environ.get("T1_SKIP_CUDA", "0") != "1":
    ce = cuda_extension()
    if ce is not None:
        exts.append(ce)
        if os.environ.get("T1_BUILD_CHECKED", "0") == "1":
            exts.append(cuda_extension(checked=True))

setup(
    name="test1_b200",
    version="0.1.0",
    packages=["test1_b200"],
    ext_modules=exts,
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
)
