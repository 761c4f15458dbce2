"""NVLink counter reader against a fake NVML (no GPU): link discovery, field fallback, unit scaling,
per-link sums and the unsupported cases."""
from types import SimpleNamespace

from deepep_slingshot_b200.utils.nvlink_counters import (FI_RCV_BYTES, FI_THROUGHPUT_RX, FI_THROUGHPUT_TX,
                                                          FI_XMIT_BYTES, NvlinkCounters, Traffic)


class FakeNvml:
    def __init__(self, active_links, supported_fields, counters):
        self.active = set(active_links)
        self.supported = set(supported_fields)
        self.counters = counters  # {(field, link): value}
        self.calls = []

    def nvmlDeviceGetHandleByIndex(self, i):
        if i != 0:
            raise RuntimeError('no such device')
        return 'h0'

    def nvmlDeviceGetNvLinkState(self, handle, link):
        if link >= 18:
            raise RuntimeError('bad link')
        return 1 if link in self.active else 0

    def nvmlDeviceGetFieldValues(self, handle, ids):
        self.calls.append(list(ids))
        out = []
        for fid, link in ids:
            ok = fid in self.supported
            out.append(SimpleNamespace(nvmlReturn=0 if ok else 3,
                                       value=SimpleNamespace(ullVal=self.counters.get((fid, link), 0))))
        return out


def test_sums_active_links_in_bytes():
    c = {(FI_XMIT_BYTES, 0): 100, (FI_XMIT_BYTES, 2): 50, (FI_RCV_BYTES, 0): 7, (FI_RCV_BYTES, 2): 3,
         (FI_XMIT_BYTES, 1): 10 ** 9}  # link 1 is down: never summed
    nv = FakeNvml([0, 2], [FI_XMIT_BYTES, FI_RCV_BYTES], c)
    r = NvlinkCounters(0, nvml=nv)
    assert r.supported and r.links == [0, 2]
    assert r.read() == Traffic(150, 10)
    nv.counters[(FI_XMIT_BYTES, 0)] += 1000
    nv.counters[(FI_RCV_BYTES, 2)] += 24
    assert r.read() - Traffic(150, 10) == Traffic(1000, 24)


def test_falls_back_to_throughput_fields_in_kib():
    c = {(FI_THROUGHPUT_TX, 5): 3, (FI_THROUGHPUT_RX, 5): 4}
    r = NvlinkCounters(0, nvml=FakeNvml([5], [FI_THROUGHPUT_TX, FI_THROUGHPUT_RX], c))
    assert r.supported
    assert r.read() == Traffic(3 * 1024, 4 * 1024)


def test_unsupported_cases_read_none():
    assert NvlinkCounters(0, nvml=FakeNvml([], [FI_XMIT_BYTES, FI_RCV_BYTES], {})).read() is None  # no links
    assert NvlinkCounters(0, nvml=FakeNvml([0], [], {})).read() is None                           # no fields
    assert NvlinkCounters(1, nvml=FakeNvml([0], [FI_XMIT_BYTES, FI_RCV_BYTES], {})).read() is None  # bad device


def test_only_reads():
    """The reader calls no NVML function that changes state (reset / freeze of counters)."""
    nv = FakeNvml([0], [FI_XMIT_BYTES, FI_RCV_BYTES], {})
    r = NvlinkCounters(0, nvml=nv)
    r.read()
    import deepep_slingshot_b200.utils.nvlink_counters as mod
    src = open(mod.__file__).read()
    assert 'nvmlDeviceResetNvLinkUtilizationCounter(' not in src and 'nvmlDeviceFreezeNvLinkUtilizationCounter(' not in src
