"""Host models of device logic (CPU): compiles tests/host_models/host_models.cu with nvcc for the host
and runs it. It drives the same __host__ __device__ scheduling and LogFMT helpers the kernels use,
and a randomized model of the pipeline-ring credit protocol."""
import os
import shutil
import subprocess

import pytest

HERE = os.path.dirname(os.path.abspath(__file__))


def test_host_models(tmp_path):
    nvcc = shutil.which('nvcc') or ('/usr/local/cuda/bin/nvcc' if os.path.exists('/usr/local/cuda/bin/nvcc') else None)
    if nvcc is None:
        pytest.skip('nvcc not available')
    exe = str(tmp_path / 'host_models')
    subprocess.run([nvcc, '-std=c++17', '-O2', '-Wno-deprecated-gpu-targets', '-o', exe,
                    os.path.join(HERE, 'host_models', 'host_models.cu')], check=True, capture_output=True, timeout=300)
    out = subprocess.run([exe], capture_output=True, text=True, timeout=300)
    assert out.returncode == 0 and 'ALL OK' in out.stdout, out.stdout + out.stderr
