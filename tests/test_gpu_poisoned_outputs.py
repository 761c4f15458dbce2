"""Initialisation check without compute-sanitizer: the normal-mode dispatch / combine tests rerun with
DEEPEP_B200_POISON_OUTPUTS=1, so every output byte starts as 0xFF (NaN for floats, -1 for ids) and a
row the kernels fail to write breaks the byte-for-byte comparison with the torch oracle.
"""
import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.mark.parametrize('target', ['tests/test_gpu_intranode.py::test_intranode_dispatch_combine',
                                    'tests/test_gpu_edge_cases.py', 'tests/test_gpu_elastic.py'])
def test_outputs_fully_written(target):
    env = dict(os.environ, DEEPEP_B200_POISON_OUTPUTS='1')
    out = subprocess.run([sys.executable, '-m', 'pytest', '-x', '-q', target], cwd=ROOT, env=env, capture_output=True,
                         text=True, timeout=1200)
    assert out.returncode == 0, out.stdout[-4000:] + out.stderr[-2000:]
