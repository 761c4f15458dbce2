"""Kernel variant table (`utils/variants.py`, written by the build): the ptxas log parser on a
synthetic log, and, once the extension is built, that every `__global__` kernel of the sources has
an entry with resources, a selection rule and no spill."""
import glob
import os
import re

import pytest

from deepep_slingshot_b200.utils import variants

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CSRC = os.path.join(ROOT, 'deepep_slingshot_b200', 'csrc')

LOG = """[1/2] /usr/local/cuda/bin/nvcc -MD -c -c /x/csrc/kernels/a.cu -o /x/build/a.o -gencode arch=compute_100a,code=sm_100a
ptxas info    : Compiling entry function '_ZN2ep8k_kernelEi' for 'sm_100a'
ptxas info    : Function properties for _ZN2ep8k_kernelEi
    8 bytes stack frame, 0 bytes spill stores, 0 bytes spill loads
ptxas info    : Used 40 registers, used 1 barriers, 128 bytes smem
ptxas info    : Function properties for _ZN2ep6helperEv
    0 bytes stack frame, 4 bytes spill stores, 4 bytes spill loads
[2/2] /usr/local/cuda/bin/nvcc -MD -c -c /x/csrc/kernels/b.cu -o /x/build/b.o
ptxas info    : Compiling entry function '_ZN2ep8m_kernelEv' for 'sm_100a'
ptxas info    : Function properties for _ZN2ep8m_kernelEv
    0 bytes stack frame, 0 bytes spill stores, 0 bytes spill loads
ptxas info    : Used 12 registers
"""


def test_parse_ptxas_log():
    t = variants.parse_ptxas(LOG, '/x/csrc')
    assert set(t) == {'kernels/a.cu', 'kernels/b.cu'}
    (a,) = t['kernels/a.cu']
    assert a == {'mangled': '_ZN2ep8k_kernelEi', 'arch': 'sm_100a', 'stack': 8, 'spill_stores': 0, 'spill_loads': 0,
                 'registers': 40, 'barriers': 1, 'smem_static': 128}
    (b,) = t['kernels/b.cu']
    assert b['registers'] == 12 and b['barriers'] == 0 and b['smem_static'] == 0  # non-entry functions ignored


def test_base_name():
    assert variants.base_name('void ep::grouped_gemm_fp8_kernel<256>(CUtensorMap_st, ep::GemmArgs)') == 'grouped_gemm_fp8_kernel'
    assert variants.base_name('ep::dispatch_pull_kernel(ep::PullArgs)') == 'dispatch_pull_kernel'


def _global_kernels():
    names = set()
    for path in glob.glob(os.path.join(CSRC, '**', '*.cu'), recursive=True):
        src = open(path).read()
        # launch bounds may hold one level of parentheses: __launch_bounds__((2 + kEpi) * 32, 1)
        for m in re.finditer(r'__global__\s+(?:void\s+)?(?:__launch_bounds__\((?:[^()]|\([^()]*\))*\)\s+)?(?:void\s+)?(\w+)\s*\(', src):
            names.add(m.group(1))
    return names


def test_every_kernel_is_in_the_built_table():
    if not os.path.exists(variants.TABLE):
        pytest.skip('the extension has not been built here (kernel_variants.json is written by setup.py)')
    rows = variants.load()
    built = {r['base'] for r in rows}
    missing = _global_kernels() - built
    assert not missing, f'kernels without a build record: {sorted(missing)}'
    for r in rows:
        assert r['arch'] == 'sm_100a' and r.get('registers', 0) > 0, r
        assert r.get('spill_stores', 0) == 0 and r.get('spill_loads', 0) == 0, r
        assert r['selected_by'], f"no selection rule for {r['base']}"
