"""Builds the sm_100a extension in-tree: ``python setup.py build_ext --inplace``.

Produces ``h3_a100/_C.*.so``.  Only ``sm_100a`` code is generated (tcgen05,
TMA and TMEM instructions exist only there).
"""

import os

os.environ.setdefault("TORCH_CUDA_ARCH_LIST", "10.0a")

from setuptools import setup  # noqa: E402
from torch.utils.cpp_extension import BuildExtension, CUDAExtension  # noqa: E402

ROOT = os.path.dirname(os.path.abspath(__file__))
SOURCES = [
    "csrc/bindings.cpp",
    "csrc/gemm/gemm_tcgen05.cu",
    "csrc/elementwise/elementwise.cu",
    "csrc/attn/attention_fwd.cu",
    "csrc/attn/attention_bwd.cu",
    "csrc/noalloc/dmd_loss_noalloc.cu",
    "csrc/comm/p2p.cu",
    "csrc/staging/pinned_pool.cpp",
]
NVCC_FLAGS = [
    "-O3",
    "-std=c++17",
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo",
    "--expt-relaxed-constexpr",
    "-Xptxas", "-v" if os.environ.get("H3_PTXAS_VERBOSE") else "-O3",
]

EXTENSIONS = [
    CUDAExtension(
        name="h3_a100._C",
        sources=[os.path.join(ROOT, s) for s in SOURCES],
        include_dirs=[os.path.join(ROOT, "csrc")],
        extra_compile_args={"cxx": ["-O3", "-std=c++17"], "nvcc": NVCC_FLAGS},
    )
]
# H3_CHECKED_BUILD=1 also builds h3_a100._C_checked: the same kernels with
# -DH3_BOUNDS_CHECK, where every global access whose index arithmetic is this
# code's own is checked against its allocation and, if outside, skipped and
# reported in the status word (tests/test_checked_build.py).
CHECKED_SOURCES = [
    "csrc/checked/checked_bindings.cpp",
    "csrc/checked/checked_gemm_tcgen05.cu",
    "csrc/checked/checked_elementwise.cu",
    "csrc/checked/checked_attention_fwd.cu",
    "csrc/checked/checked_attention_bwd.cu",
    "csrc/checked/checked_p2p.cu",
    "csrc/checked/checked_pinned_pool.cpp",
]
if os.environ.get("H3_CHECKED_BUILD", "0") == "1":
    EXTENSIONS.append(
        CUDAExtension(
            name="h3_a100._C_checked",
            sources=[os.path.join(ROOT, s) for s in CHECKED_SOURCES],
            include_dirs=[os.path.join(ROOT, "csrc")],
            extra_compile_args={"cxx": ["-O3", "-std=c++17", "-DH3_BOUNDS_CHECK"],
                                "nvcc": NVCC_FLAGS + ["-DH3_BOUNDS_CHECK"]},
        )
    )

setup(
    name="h3_a100_b200_ext",
    ext_modules=EXTENSIONS,
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
)
