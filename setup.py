"""Build of the sm_100a extension `deepep_slingshot_b200._C` (in-tree: `python setup.py build_ext --inplace`).

Only Blackwell datacenter parts are targeted: every CUDA translation unit is compiled with
`-gencode arch=compute_100a,code=sm_100a`, which also keeps torch from adding its own arch list.
A kernel that spills registers fails the build (ptxas --warn-on-spills --warning-as-error).
"""
import os
from setuptools import setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension

ROOT = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join("deepep_slingshot_b200", "csrc")

SOURCES = [
    os.path.join(CSRC, "python_api.cpp"),
    os.path.join(CSRC, "runtime", "buffer.cpp"),
    os.path.join(CSRC, "runtime", "ops.cpp"),
    os.path.join(CSRC, "runtime", "symmetric.cpp"),
    os.path.join(CSRC, "kernels", "intranode.cu"),
    os.path.join(CSRC, "kernels", "low_latency.cu"),
    os.path.join(CSRC, "kernels", "quant.cu"),
    os.path.join(CSRC, "kernels", "permute.cu"),
    os.path.join(CSRC, "kernels", "permute_noalloc.cu"),
    os.path.join(CSRC, "kernels", "gemm_sm100.cu"),
    os.path.join(CSRC, "kernels", "gemm_bf16_sm100.cu"),
    os.path.join(CSRC, "kernels", "gemm_masked_sm100.cu"),
    os.path.join(CSRC, "kernels", "fused_dispatch_gemm.cu"),
    os.path.join(CSRC, "kernels", "symmetric_ops.cu"),
    os.path.join(CSRC, "kernels", "transport_checks.cu"),
    os.path.join(CSRC, "kernels", "moe_backward.cu"),
]

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo", "-O3", "-std=c++17",
    "--expt-relaxed-constexpr",
    "-Xptxas", "-v",
    # Build-time gate on register spills (the reference's JIT fails a kernel that uses local memory
    # for spills): ptxas turns a spill warning into a build error.
    "-Xptxas", "--warn-on-spills",
    "-Xptxas", "--warning-as-error",
    "--diag-suppress=177,550",
]
CXX_FLAGS = ["-O3", "-std=c++17", "-Wno-unused-function"]

setup(
    name="deepep_slingshot_b200",
    version="0.1.0",
    packages=["deepep_slingshot_b200"],
    ext_modules=[
        CUDAExtension(
            name="deepep_slingshot_b200._C",
            sources=SOURCES,
            include_dirs=[os.path.join(ROOT, CSRC)],
            extra_compile_args={"cxx": CXX_FLAGS, "nvcc": NVCC_FLAGS},
        )
    ],
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
)
