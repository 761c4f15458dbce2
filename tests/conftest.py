import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

# Tests of kernels that have not run on a B200 yet; they move into tests/ after their first GPU run.
# DEEPEP_B200_RUN_PENDING=1 collects them (python -m pytest tests/pending -m gpu).
collect_ignore = [] if os.environ.get('DEEPEP_B200_RUN_PENDING') == '1' else ['pending']
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line('markers', 'gpu: needs a CUDA GPU (B200, sm_100a)')
    config.addinivalue_line('markers', 'multigpu: needs two or more GPUs of one NVLink domain')
