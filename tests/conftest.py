import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line('markers', 'gpu: needs a CUDA GPU (B200, sm_100a)')
    config.addinivalue_line('markers', 'multigpu: needs two or more GPUs of one NVLink domain')


def pytest_sessionfinish(session, exitstatus):
    """Report (and end) anything that would keep the interpreter from exiting: child processes this
    session spawned that are still alive (multiprocessing joins them at exit) and non-daemon threads."""
    import multiprocessing
    import threading
    for child in multiprocessing.active_children():
        sys.stderr.write(f'\n[conftest] child process {child.pid} ({child.name}) still alive at session end: killing it\n')
        child.kill()
        child.join(timeout=10)
    for t in threading.enumerate():
        if t is not threading.main_thread() and not t.daemon:
            sys.stderr.write(f'\n[conftest] non-daemon thread still running at session end: {t.name}\n')
