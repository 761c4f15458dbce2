"""Process-group bootstrap and topology helpers.

Parity with the reference's `deep_ep/utils/envs.py:74-268` (`init_dist`, NVLink checks,
`get_nvlink_gbs`). Rendezvous defaults to 127.0.0.1. NVLink bandwidth comes from NVML when
available; the fallback is the B200 measured peer-copy figure (770 GB/s per direction).
"""
import os
import subprocess
from typing import Optional, Tuple

import torch
import torch.distributed as dist

B200_NVLINK_GBS = 770.0  # measured peer copy per direction on this pool (nominal 900)


def init_dist(local_rank: Optional[int] = None, num_local_ranks: Optional[int] = None, backend: str = 'nccl',
              timeout_s: int = 120) -> Tuple[int, int, dist.ProcessGroup]:
    """Initialise torch.distributed from torchrun/env variables; returns (rank, world_size, group)."""
    import datetime
    os.environ.setdefault('MASTER_ADDR', '127.0.0.1')
    os.environ.setdefault('MASTER_PORT', '29577')
    if local_rank is None:
        local_rank = int(os.environ.get('LOCAL_RANK', 0))
    world = int(os.environ.get('WORLD_SIZE', num_local_ranks or 1))
    rank = int(os.environ.get('RANK', local_rank))
    kwargs = dict(backend=backend, world_size=world, rank=rank, timeout=datetime.timedelta(seconds=timeout_s))
    if backend == 'nccl':
        torch.cuda.set_device(local_rank)
        kwargs['device_id'] = torch.device('cuda', local_rank)
    if not dist.is_initialized():
        dist.init_process_group(**kwargs)
    return dist.get_rank(), dist.get_world_size(), dist.new_group(list(range(world)))


def check_nvlink_connections(group: Optional[dist.ProcessGroup]) -> None:
    """All ranks of an EP group must be NVLink peers (one box): checked through CUDA peer access."""
    if group is None or not torch.cuda.is_available():
        return
    n = torch.cuda.device_count()
    dev = torch.cuda.current_device()
    for other in range(n):
        if other != dev and not torch.cuda.can_device_access_peer(dev, other):
            raise RuntimeError(f'GPU {dev} cannot access GPU {other} as a peer; the EP group must be one NVLink domain')


def get_nvlink_gbs() -> float:
    """Per-direction NVLink bandwidth of this GPU in GB/s (NVML link count x per-link rate)."""
    try:
        import pynvml
        pynvml.nvmlInit()
        h = pynvml.nvmlDeviceGetHandleByIndex(torch.cuda.current_device() if torch.cuda.is_available() else 0)
        links = 0
        for i in range(18):
            try:
                if pynvml.nvmlDeviceGetNvLinkState(h, i) == pynvml.NVML_FEATURE_ENABLED:
                    links += 1
            except pynvml.NVMLError:
                break
        pynvml.nvmlShutdown()
        if links > 0:
            return min(links * 50.0, 900.0) * (B200_NVLINK_GBS / 900.0)
    except Exception:
        pass
    return B200_NVLINK_GBS


def get_rdma_gbs() -> float:
    """No RDMA fabric inside one NVLink box."""
    return 0.0


def nvidia_smi_clocks() -> Optional[str]:
    """One `nvidia-smi` sample (current and maximum SM clock) of the current CUDA device, named by
    its PCI bus id so that CUDA_VISIBLE_DEVICES does not matter; None without nvidia-smi."""
    from .numa import pci_bus_id
    dev = pci_bus_id(torch.cuda.current_device()) if torch.cuda.is_available() else None
    try:
        return subprocess.check_output(['nvidia-smi', '--query-gpu=clocks.sm,clocks.max.sm', '--format=csv,noheader'] +
                                       (['-i', dev] if dev else []), text=True, timeout=10)
    except Exception:
        return None


_SEEDS = {'local': None, 'global': None}


def init_seed(global_seed: int) -> None:
    """Seed torch / random with `global_seed + rank` (the local seed) for reproducible runs."""
    import random
    rank = dist.get_rank() if dist.is_initialized() else 0
    _SEEDS['global'], _SEEDS['local'] = global_seed, global_seed + rank
    torch.manual_seed(global_seed + rank)
    random.seed(global_seed + rank)


def get_local_seed() -> Optional[int]:
    """The seed of this rank set by `init_seed` (None before)."""
    return _SEEDS['local']


def get_global_seed() -> Optional[int]:
    """The global seed set by `init_seed` (None before)."""
    return _SEEDS['global']


def dist_print(s: str = '', once_in_node: bool = False) -> None:
    """Print from every rank (or only local rank 0 with `once_in_node`), then barrier."""
    local_rank = int(os.environ.get('LOCAL_RANK', dist.get_rank() if dist.is_initialized() else 0))
    if not once_in_node or local_rank == 0:
        print(s, flush=True)
    if dist.is_initialized():
        dist.barrier()


def get_physical_domain_size(group: dist.ProcessGroup) -> Tuple[int, int]:
    """(RDMA ranks, NVLink ranks): one NVLink domain here."""
    return 1, group.size()


def get_logical_domain_size(group: dist.ProcessGroup, allow_hybrid_mode: bool = True) -> Tuple[int, int]:
    """(scale-out ranks, scale-up ranks): one NVLink domain here."""
    return 1, group.size()


def check_torch_deterministic() -> None:
    """Deterministic algorithms together with `fill_uninitialized_memory` make `torch.empty` launch an
    initialisation kernel that can overlap with communication: refuse that combination."""
    import torch.utils.deterministic
    assert not (torch.are_deterministic_algorithms_enabled() and torch.utils.deterministic.fill_uninitialized_memory)


def check_fast_rdma_atomic_support(nic_name: str = 'mlx5_0') -> bool:
    """Whether the named RDMA NIC supports fast atomics (the reference sizes its QP count with it,
    [DE]deep_ep/utils/envs.py:223, [DE]deep_ep/buffers/elastic.py:203). One NVLink box has no RDMA
    transport in this library, so the answer only reports what `ibstat` says and nothing here
    depends on it; False without `ibstat` or without the NIC."""
    import subprocess
    try:
        out = subprocess.run(['ibstat', nic_name], capture_output=True, text=True, timeout=10)
    except (OSError, subprocess.TimeoutExpired):
        return False
    if out.returncode != 0:
        return False
    # ConnectX-7 (MT4129) and older lack them; MT4131 (ConnectX-8) and newer have them.
    for line in out.stdout.splitlines():
        line = line.strip()
        if line.startswith('CA type:') and 'MT' in line:
            try:
                return int(line.split('MT')[-1].strip()) >= 4131
            except ValueError:
                return False
    return False
