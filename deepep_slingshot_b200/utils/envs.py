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
    try:
        return subprocess.check_output(['nvidia-smi', '--query-gpu=clocks.sm,clocks.max.sm', '--format=csv,noheader'],
                                       text=True, timeout=10)
    except Exception:
        return None
