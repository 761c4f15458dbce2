"""Build of the sm_100a extension `deepep_slingshot_b200._C` (in-tree: `python setup.py build_ext --inplace`).

Only Blackwell datacenter parts are targeted: every CUDA translation unit is compiled with
`-gencode arch=compute_100a,code=sm_100a`, which also keeps torch from adding its own arch list.
A kernel that spills registers fails the build (ptxas --warn-on-spills --warning-as-error), and
every kernel entry's resource use (registers, shared memory, stack, spills per template instance)
is recorded in `deepep_slingshot_b200/kernel_variants.json` (`utils/variants.py` reads it).
"""
import json
import os
import re
import subprocess
import sys
import tempfile

from setuptools import setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension

ROOT = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join("deepep_slingshot_b200", "csrc")

SOURCES = [
    os.path.join(CSRC, "python_api.cpp"),
    os.path.join(CSRC, "runtime", "buffer.cpp"),
    os.path.join(CSRC, "runtime", "ops.cpp"),
    os.path.join(CSRC, "runtime", "symmetric.cpp"),
    os.path.join(CSRC, "runtime", "host_segment.cpp"),
    os.path.join(CSRC, "kernels", "intranode.cu"),
    os.path.join(CSRC, "kernels", "low_latency.cu"),
    os.path.join(CSRC, "kernels", "quant.cu"),
    os.path.join(CSRC, "kernels", "permute.cu"),
    os.path.join(CSRC, "kernels", "permute_noalloc.cu"),
    os.path.join(CSRC, "kernels", "gemm_sm100.cu"),
    os.path.join(CSRC, "kernels", "gemm_bf16_sm100.cu"),
    os.path.join(CSRC, "kernels", "gemm_masked_sm100.cu"),
    os.path.join(CSRC, "kernels", "gemm_combine.cu"),
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

VARIANT_TABLE = os.path.join(ROOT, "deepep_slingshot_b200", "kernel_variants.json")


def _variants_module():
    """`deepep_slingshot_b200/utils/variants.py` loaded by path (the package itself imports the
    extension that is being built)."""
    import importlib.util
    spec = importlib.util.spec_from_file_location("_ep_variants", os.path.join(ROOT, "deepep_slingshot_b200", "utils", "variants.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def demangle(names):
    try:
        res = subprocess.run(["c++filt"], input="\n".join(names), capture_output=True, text=True, timeout=60)
        lines = res.stdout.splitlines()
        if res.returncode == 0 and len(lines) == len(names):
            return lines
    except (OSError, subprocess.TimeoutExpired):
        pass
    return list(names)


def write_variant_table(log: str) -> None:
    """Merge this build's per-kernel resource records into the package's kernel variant table (an
    incremental build recompiles only some translation units; the others keep their records)."""
    table = {}
    if os.path.exists(VARIANT_TABLE):
        with open(VARIANT_TABLE) as f:
            table = json.load(f)
    by_source = table.get("sources", {})
    fresh = _variants_module().parse_ptxas(log, os.path.join(ROOT, CSRC))
    for src, entries in fresh.items():
        names = demangle([e["mangled"] for e in entries])
        for e, n in zip(entries, names):
            e["name"] = n
        by_source[src] = entries
    table = {"arch": "sm_100a", "nvcc_flags": NVCC_FLAGS, "sources": dict(sorted(by_source.items()))}
    with open(VARIANT_TABLE, "w") as f:
        json.dump(table, f, indent=1)


class BuildWithVariantTable(BuildExtension):
    """The extension build, with its compiler output captured and the ptxas resource lines of every
    kernel entry written to `deepep_slingshot_b200/kernel_variants.json` (registers, shared memory,
    stack and spills per template instance), then echoed."""

    def build_extensions(self):
        sys.stdout.flush()
        sys.stderr.flush()
        with tempfile.TemporaryFile() as log:
            saved_out, saved_err = os.dup(1), os.dup(2)
            os.dup2(log.fileno(), 1)
            os.dup2(log.fileno(), 2)
            failed = None
            try:
                super().build_extensions()
            except BaseException as exc:  # re-raised after the output is restored
                failed = exc
            finally:
                sys.stdout.flush()
                sys.stderr.flush()
                os.dup2(saved_out, 1)
                os.dup2(saved_err, 2)
                os.close(saved_out)
                os.close(saved_err)
            log.seek(0)
            text = log.read().decode(errors="replace")
        sys.stdout.write(text)
        sys.stdout.flush()
        if failed is not None:
            raise failed
        write_variant_table(text)


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
            extra_link_args=["-lrt"],  # shm_open / shm_unlink (host segments)
        )
    ],
    cmdclass={"build_ext": BuildWithVariantTable.with_options(use_ninja=True)},
)
