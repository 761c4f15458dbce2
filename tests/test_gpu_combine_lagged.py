"""GPU test of the combine with lagged arrival announcements (DEEPEP_B200_COMBINE_ANNOUNCE=lagged):
the normal-mode dispatch/combine tests, run in a child process with the knob set (the runtime reads
it when a buffer is built).
"""
import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.mark.parametrize('target', ['tests/test_gpu_intranode.py::test_intranode_dispatch_combine',
                                    'tests/test_gpu_intranode.py::test_intranode_deepseek_shape'])
def test_combine_lagged_announcements(target):
    env = dict(os.environ, DEEPEP_B200_COMBINE_ANNOUNCE='lagged')
    out = subprocess.run([sys.executable, '-m', 'pytest', '-x', '-q', target], cwd=ROOT, env=env, capture_output=True,
                         text=True, timeout=900)
    assert out.returncode == 0, out.stdout[-4000:] + out.stderr[-2000:]
