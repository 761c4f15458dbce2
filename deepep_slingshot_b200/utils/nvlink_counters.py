"""NVLink traffic counters of one GPU, read through NVML (read-only).

The NVLink transport moves bytes with peer loads and stores issued by kernels, which no profiler of a
single process attributes to links. The GPU's own per-link counters do: NVML exposes, per NVLink,
the data bytes transmitted and received (`NVML_FI_DEV_NVLINK_COUNT_XMIT_BYTES` /
`..._RCV_BYTES`, field ids 202 / 204, scope = link id), and on older drivers the data throughput
counters in KiB (`..._THROUGHPUT_DATA_TX` / `_RX`, 138 / 139). Reading them around a timed region
gives the bytes that actually crossed this GPU's links, to set beside the algorithmic byte count of
a benchmark (the reference checks its transport's byte accounting against NIC counters in its
qualification harness; here the counters are NVLink's).

Only reads: no counter is reset or frozen (`nvmlDeviceResetNvLinkUtilizationCounter` and the
freeze calls change device state and are never called).

    c = NvlinkCounters(device_index)
    before = c.read()
    ... timed region ...
    moved = c.read() - before     # Traffic(tx_bytes, rx_bytes), or None when unsupported
"""
from dataclasses import dataclass
from typing import List, Optional, Tuple

FI_XMIT_BYTES, FI_RCV_BYTES = 202, 204          # bytes, per link
FI_THROUGHPUT_TX, FI_THROUGHPUT_RX = 138, 139   # KiB, per link (older drivers)
MAX_LINKS = 18
NVML_SUCCESS = 0


@dataclass(frozen=True)
class Traffic:
    tx_bytes: int
    rx_bytes: int

    def __sub__(self, other: 'Traffic') -> 'Traffic':
        return Traffic(self.tx_bytes - other.tx_bytes, self.rx_bytes - other.rx_bytes)


def _load_nvml():
    try:
        import pynvml
    except ImportError:
        return None
    try:
        pynvml.nvmlInit()
    except Exception:  # no driver (CPU host) or NVML failure
        return None
    return pynvml


class NvlinkCounters:
    """Sum of the per-link NVLink data counters of one GPU (`nvml` may be a stand-in module for tests)."""

    def __init__(self, device_index: int, nvml=None) -> None:
        self.nvml = nvml if nvml is not None else _load_nvml()
        self.handle = None
        self.links: List[int] = []
        self.fields: Optional[Tuple[int, int, int]] = None  # (tx id, rx id, bytes per unit)
        if self.nvml is None:
            return
        try:
            self.handle = self.nvml.nvmlDeviceGetHandleByIndex(device_index)
        except Exception:
            self.handle = None
            return
        self.links = [l for l in range(MAX_LINKS) if self._link_active(l)]
        for tx, rx, unit in ((FI_XMIT_BYTES, FI_RCV_BYTES, 1), (FI_THROUGHPUT_TX, FI_THROUGHPUT_RX, 1024)):
            if self.links and self._values([(tx, self.links[0]), (rx, self.links[0])]) is not None:
                self.fields = (tx, rx, unit)
                break

    def _link_active(self, link: int) -> bool:
        try:
            return bool(self.nvml.nvmlDeviceGetNvLinkState(self.handle, link))
        except Exception:
            return False

    def _values(self, ids) -> Optional[List[int]]:
        try:
            vals = self.nvml.nvmlDeviceGetFieldValues(self.handle, ids)
        except Exception:
            return None
        out = []
        for v in vals:
            if v.nvmlReturn != NVML_SUCCESS:
                return None
            out.append(int(v.value.ullVal))
        return out

    @property
    def supported(self) -> bool:
        return self.fields is not None

    def read(self) -> Optional[Traffic]:
        """Total data bytes sent and received over this GPU's active links so far (None if unsupported)."""
        if self.fields is None:
            return None
        tx_id, rx_id, unit = self.fields
        vals = self._values([(tx_id, l) for l in self.links] + [(rx_id, l) for l in self.links])
        if vals is None:
            return None
        n = len(self.links)
        return Traffic(sum(vals[:n]) * unit, sum(vals[n:]) * unit)
