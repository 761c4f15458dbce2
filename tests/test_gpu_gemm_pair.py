"""GPU test of the FP8 grouped GEMM on CTA pairs (`cta_group::2`, 256 x 256 tiles,
DEEPEP_B200_GEMM_PAIR=1), against the fp32 oracle of `tests/test_gpu_gemm.py`: experts with an odd
number of 128-row m-tiles (the second CTA of the last pair computes rows it must not store), empty
experts, partial tiles, and the DeepSeek-V3 shapes. The switch is read once per process, so the
cases run in a child process. DEEPEP_B200_GEMM_PAIR=2 selects the variant with eight epilogue warps
and the pipelined promotion.
"""
import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

_CHILD = r'''
import torch
from tests.test_gpu_gemm import test_grouped_gemm_fp8
for counts, n, k in [([200, 0, 130, 37], 256, 256), ([300, 257, 1, 640], 512, 1024), ([128], 256, 128),
                     ([1000, 900, 1100, 512, 64, 700, 333, 800], 4096, 7168), ([1024] * 4, 7168, 2048),
                     ([129, 385, 0, 1], 128, 256)]:   # n = 128 falls back to one-CTA tiles
    test_grouped_gemm_fp8(counts, n, k)
print("PAIR OK")
'''


@pytest.mark.parametrize('variant', ['1', '2'])
def test_grouped_gemm_fp8_cta_pairs(variant):
    env = dict(os.environ, DEEPEP_B200_GEMM_PAIR=variant, PYTHONPATH=ROOT)
    out = subprocess.run([sys.executable, '-c', _CHILD], cwd=ROOT, env=env, capture_output=True, text=True, timeout=600)
    assert out.returncode == 0 and 'PAIR OK' in out.stdout, out.stdout[-3000:] + out.stderr[-3000:]
