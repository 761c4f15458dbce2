"""CPU tests of the package locator (`utils/find_pkgs.py`) against fake distributions, and of the
communicator handles (`utils/comm.py`) against fake process-group backends."""
import os
import sys
from types import SimpleNamespace

import pytest

from deepep_slingshot_b200.utils import comm, find_pkgs


class FakeFile:
    def __init__(self, path):
        self.path = path

    def __str__(self):
        return self.path

    def locate(self):
        return self.path


def fake_dist(name, site, files):
    return SimpleNamespace(metadata={'Name': name}, _path=os.path.join(site, name.replace('-', '_') + '.dist-info'),
                           files=[FakeFile(f) for f in files])


def test_env_var_wins(monkeypatch):
    monkeypatch.setenv('DEEPEP_B200_NCCL_ROOT_DIR', '/opt/my-nccl')
    assert find_pkgs.find_pkg_root('nccl', 'libnccl.so', dists=[]) == '/opt/my-nccl'


def test_wheel_lookup_prefers_sys_path_order(monkeypatch):
    monkeypatch.delenv('DEEPEP_B200_NCCL_ROOT_DIR', raising=False)
    monkeypatch.delenv('NCCL_DIR', raising=False)
    first, second = sys.path[0], '/nowhere/site-packages'
    d_late = fake_dist('nvidia-nccl-cu12', second, [f'{second}/nvidia/nccl/lib/libnccl.so.2'])
    d_early = fake_dist('nvidia-nccl-cu12', first, [f'{first}/nvidia/nccl/lib/libnccl.so.2'])
    other = fake_dist('nvidia-cublas-cu12', first, [f'{first}/nvidia/cublas/lib/libcublas.so.12'])
    root = find_pkgs.find_pkg_root('nccl', 'libnccl.so', dists=[d_late, other, d_early])
    assert root == f'{first}/nvidia/nccl'


def test_missing_package(monkeypatch):
    monkeypatch.delenv('DEEPEP_B200_NVSHMEM_ROOT_DIR', raising=False)
    monkeypatch.delenv('NVSHMEM_DIR', raising=False)
    assert find_pkgs.find_pkg_root('nvshmem', 'libnvshmem', optional=True, dists=[]) is None
    with pytest.raises(FileNotFoundError):
        find_pkgs.find_pkg_root('nvshmem', 'libnvshmem', dists=[])


def test_installed_nccl_is_found_when_present():
    root = find_pkgs.find_nccl_root(optional=True)
    if root is not None:
        assert os.path.isdir(root)


class FakeBackend:
    def __init__(self, ptr):
        self.ptr = ptr

    def _comm_ptr(self):
        return self.ptr


class FakeGroup:
    def __init__(self, backend):
        self.backend = backend

    def _get_backend(self, device):
        if self.backend is None:
            raise RuntimeError('no backend for cuda')
        return self.backend


def test_comm_handle_is_cached_and_unmanaged():
    comm.destroy_all_managed_nccl_comm()
    g = FakeGroup(FakeBackend(0x1234))
    h = comm.get_nccl_comm_handle(g)
    assert h.get() == 0x1234 and not h.managed
    assert comm.get_nccl_comm_handle(g) is h
    comm.destroy_all_managed_nccl_comm()
    assert comm.get_nccl_comm_handle(g) is not h


def test_comm_handle_errors():
    with pytest.raises(RuntimeError):
        comm.get_nccl_comm_handle(FakeGroup(None))
    with pytest.raises(RuntimeError):
        comm.get_nccl_comm_handle(FakeGroup(SimpleNamespace()))
    with pytest.raises(ValueError):
        comm.NCCLCommHandle(1, managed=True)
