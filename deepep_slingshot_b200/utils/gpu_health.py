"""Read-only GPU health snapshot through NVML, for the qualification ladder's resume step.

The reference's gate controller resumes after a failed gate only with a recorded reason and after a
GPU health check (its controller runs `nvidia-smi` before it continues). Here the check reads, per
visible GPU, what says the device itself is unwell rather than the workload:
  * uncorrected ECC errors since the driver loaded (volatile count);
  * pending page retirements / row remappings (a reset is needed to apply them);
  * hardware slowdown or thermal slowdown clock-event reasons active right now;
  * the GPU temperature (reported, not judged).
Every call is a query; nothing is reset, cleared or set (no clocks, no ECC mode, no persistence).
`nvml` may be a stand-in module (tests).
"""
from dataclasses import dataclass, field
from typing import List, Optional

HW_SLOWDOWN = 0x8
SW_THERMAL_SLOWDOWN = 0x20
HW_THERMAL_SLOWDOWN = 0x40


@dataclass
class GpuHealth:
    index: int
    name: str = ''
    temperature_c: Optional[int] = None
    uncorrected_ecc: Optional[int] = None
    retirement_pending: Optional[bool] = None
    remap_pending: Optional[bool] = None
    slowdown_reasons: List[str] = field(default_factory=list)

    @property
    def problems(self) -> List[str]:
        out = []
        if self.uncorrected_ecc:
            out.append(f'{self.uncorrected_ecc} uncorrected ECC errors')
        if self.retirement_pending:
            out.append('page retirement pending')
        if self.remap_pending:
            out.append('row remapping pending')
        out.extend(self.slowdown_reasons)
        return out


def _load_nvml():
    import pynvml
    pynvml.nvmlInit()
    return pynvml


def _try(fn, *args):
    try:
        return fn(*args)
    except Exception:  # the query is not supported on this device / driver
        return None


def snapshot(nvml=None) -> List[GpuHealth]:
    """Health of every GPU NVML sees (read-only queries)."""
    nv = nvml if nvml is not None else _load_nvml()
    out = []
    for i in range(nv.nvmlDeviceGetCount()):
        h = nv.nvmlDeviceGetHandleByIndex(i)
        g = GpuHealth(index=i)
        name = _try(nv.nvmlDeviceGetName, h)
        g.name = name.decode() if isinstance(name, bytes) else (name or '')
        g.temperature_c = _try(nv.nvmlDeviceGetTemperature, h, 0)  # NVML_TEMPERATURE_GPU
        g.uncorrected_ecc = _try(nv.nvmlDeviceGetTotalEccErrors, h, 1, 0)  # uncorrected, volatile
        pend = _try(nv.nvmlDeviceGetRetiredPagesPendingStatus, h)
        g.retirement_pending = None if pend is None else bool(pend)
        rows = _try(nv.nvmlDeviceGetRemappedRows, h)  # (corrected, uncorrected, pending, failure)
        g.remap_pending = None if rows is None else bool(rows[2] or rows[3])
        reasons = _try(nv.nvmlDeviceGetCurrentClocksEventReasons, h)
        if reasons is not None:
            for bit, label in ((HW_SLOWDOWN, 'hw_slowdown active'), (HW_THERMAL_SLOWDOWN, 'hw_thermal_slowdown active'),
                               (SW_THERMAL_SLOWDOWN, 'sw_thermal_slowdown active')):
                if reasons & bit:
                    g.slowdown_reasons.append(label)
        out.append(g)
    return out


def unhealthy(report: List[GpuHealth]) -> List[str]:
    """One line per GPU with a problem (empty: all healthy)."""
    return [f'GPU {g.index} ({g.name}): ' + ', '.join(g.problems) for g in report if g.problems]
