"""Host CPU placement next to a GPU, with a fake NVML (reads only) and a fake device lookup."""
import os

import pytest

from deepep_slingshot_b200.utils import numa


class FakeNvml:
    def __init__(self, words, fail=False):
        self.words, self.fail, self.calls = words, fail, []

    def nvmlInit(self):
        self.calls.append('init')

    def nvmlShutdown(self):
        self.calls.append('shutdown')

    def nvmlDeviceGetHandleByPciBusId(self, bus):
        if self.fail:
            raise RuntimeError('no such device')
        self.calls.append(bus)
        return 'h'

    def nvmlDeviceGetCpuAffinity(self, handle, words):
        self.calls.append(('affinity', words))
        return self.words[:words]


@pytest.fixture
def fake_bus(monkeypatch):
    monkeypatch.setattr(numa, 'pci_bus_id', lambda device: f'00000000:{0x18 + device:02x}:00.0')


def test_local_cpus_from_the_affinity_mask(fake_bus, monkeypatch):
    monkeypatch.setattr(os, 'sched_getaffinity', lambda pid: set(range(128)))
    nv = FakeNvml([0b1111 << 4, 1 << 3])
    cpus = numa.gpu_local_cpus(2, nvml=nv, num_cpus=128)
    assert cpus == {4, 5, 6, 7, 64 + 3}
    assert nv.calls[:2] == ['init', '00000000:1a:00.0'] and ('affinity', 2) in nv.calls and nv.calls[-1] == 'shutdown'


def test_local_cpus_limited_to_the_allowed_set(fake_bus, monkeypatch):
    monkeypatch.setattr(os, 'sched_getaffinity', lambda pid: {5, 6})
    assert numa.gpu_local_cpus(0, nvml=FakeNvml([0xff]), num_cpus=8) == {5, 6}
    monkeypatch.setattr(os, 'sched_getaffinity', lambda pid: {9})
    assert numa.gpu_local_cpus(0, nvml=FakeNvml([0xff]), num_cpus=16) is None


def test_unavailable_nvml_or_device_changes_nothing(fake_bus, monkeypatch):
    applied = []
    monkeypatch.setattr(os, 'sched_setaffinity', lambda pid, cpus: applied.append(cpus))
    assert numa.bind_process_to_gpu(0, nvml=FakeNvml([0xff], fail=True)) is None
    monkeypatch.setattr(numa, 'pci_bus_id', lambda device: None)
    assert numa.bind_process_to_gpu(0, nvml=FakeNvml([0xff])) is None
    assert applied == []


def test_bind_applies_the_local_set_and_can_be_disabled(fake_bus, monkeypatch):
    applied = []
    monkeypatch.setattr(os, 'sched_getaffinity', lambda pid: set(range(16)))
    monkeypatch.setattr(os, 'sched_setaffinity', lambda pid, cpus: applied.append(set(cpus)))
    assert numa.bind_process_to_gpu(1, nvml=FakeNvml([0x0f0])) == {4, 5, 6, 7}
    assert applied == [{4, 5, 6, 7}]
    monkeypatch.setenv('DEEPEP_B200_NUMA_BIND', '0')
    assert numa.bind_process_to_gpu(1, nvml=FakeNvml([0x0f0])) is None
    assert len(applied) == 1
