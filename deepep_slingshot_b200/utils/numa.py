"""Host CPU placement next to a GPU.

Pinned host buffers are allocated on the NUMA node of the thread that first touches them, and a
host-to-device copy from the other socket crosses the inter-socket link on the way to the GPU's PCIe
root. A process that feeds one GPU (one rank per GPU) should therefore run on, and allocate from,
the CPUs that NVML reports as local to that GPU. This module only reads from NVML
(`nvmlDeviceGetCpuAffinity`) and changes nothing on the GPU: `bind_process_to_gpu` sets this
process's own CPU affinity (`os.sched_setaffinity`), before its pinned buffers are allocated.
"""
import os
from typing import Optional, Set


def pci_bus_id(device: int) -> Optional[str]:
    """PCI bus id of CUDA device `device` in NVML / nvidia-smi form (`00000000:18:00.0`)."""
    try:
        import torch
        p = torch.cuda.get_device_properties(device)
        return f'{p.pci_domain_id:08x}:{p.pci_bus_id:02x}:{p.pci_device_id:02x}.0'
    except Exception:  # no CUDA device, or a torch without the PCI fields
        return None


def gpu_local_cpus(device: int, nvml=None, num_cpus: Optional[int] = None) -> Optional[Set[int]]:
    """CPUs NVML reports as close to CUDA device `device` (matched by PCI bus id, so the CUDA and
    NVML orderings may differ), intersected with the CPUs this process may use; None when NVML or the
    device is unavailable or the set would be empty. `nvml` defaults to the `pynvml` module."""
    bus = pci_bus_id(device)
    if bus is None:
        return None
    try:
        if nvml is None:
            import pynvml as nvml
        nvml.nvmlInit()
    except Exception:
        return None
    try:
        handle = nvml.nvmlDeviceGetHandleByPciBusId(bus)
        n = num_cpus or os.cpu_count() or 1
        words = nvml.nvmlDeviceGetCpuAffinity(handle, (n + 63) // 64)
        cpus = {64 * w + b for w, word in enumerate(words) for b in range(64) if (int(word) >> b) & 1}
    except Exception:
        return None
    finally:
        try:
            nvml.nvmlShutdown()
        except Exception:
            pass
    try:
        cpus &= os.sched_getaffinity(0)
    except (AttributeError, OSError):
        pass
    return cpus or None


def bind_process_to_gpu(device: int, nvml=None) -> Optional[Set[int]]:
    """Restrict this process to the CPUs local to CUDA device `device` (see `gpu_local_cpus`). Call it
    before allocating pinned host memory. Returns the CPU set applied, or None if nothing changed.
    `DEEPEP_B200_NUMA_BIND=0` turns it off."""
    if os.environ.get('DEEPEP_B200_NUMA_BIND', '1') == '0':
        return None
    cpus = gpu_local_cpus(device, nvml=nvml)
    if not cpus:
        return None
    try:
        os.sched_setaffinity(0, cpus)
    except (AttributeError, OSError):
        return None
    return cpus
