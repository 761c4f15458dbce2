"""GPU test of the FP8 grouped GEMM with each tile width against the same fp32 oracle: 128-wide tiles
forced (DEEPEP_B200_GEMM_BN=128) and 256-wide tiles requested explicitly (the default when N % 256 ==
0). The tile width is read once per process, so each case runs in a child process.
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
for counts, n, k in [([200, 0, 130, 37], 256, 256), ([300, 257, 1, 640], 512, 1024),
                     ([1000, 900, 1100, 512, 64, 700, 333, 800], 4096, 7168), ([128], 128, 128)]:
    test_grouped_gemm_fp8(counts, n, k)   # n = 128 always takes 128-wide tiles
print("WIDE OK")
'''


@pytest.mark.parametrize('bn', ['128', '256'])
def test_grouped_gemm_fp8_tile_widths(bn):
    env = dict(os.environ, DEEPEP_B200_GEMM_BN=bn, PYTHONPATH=ROOT)
    out = subprocess.run([sys.executable, '-c', _CHILD], cwd=ROOT, env=env, capture_output=True, text=True, timeout=600)
    assert out.returncode == 0 and 'WIDE OK' in out.stdout, out.stdout[-3000:] + out.stderr[-3000:]
