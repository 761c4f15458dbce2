"""Host-memory segments shared by the ranks of one box: the elastic API's hybrid CPU memory.

`HostSegments(group, num_bytes)` is collective: every rank creates one named POSIX shared-memory
segment of `num_bytes`, the names go around the group, and every rank maps every rank's segment
(`csrc/runtime/host_segment.cpp`). `view(rank)` is a CPU uint8 tensor over a rank's segment;
`device_ptrs()` registers the mappings with CUDA on first use and returns their device addresses,
which kernels read directly over PCIe / C2C. `ElasticBuffer(num_cpu_bytes=...)` keeps its Engram
storage here, as the reference keeps it in its CPU segments ([DE]deep_ep/buffers/elastic.py:208-213,
`create_cpu_handle` with POSIX FD handles; [DE]deep_ep/buffers/elastic.py:285-306 for the sizes).

A segment's name is unlinked when its creator destroys it; a process that dies first leaves its
name under /dev/shm (named `deepep_b200_*`) until it is removed.
"""
import secrets
from typing import List, Optional

import torch
import torch.distributed as dist

from .._ext import require_ext

NAME_PREFIX = '/deepep_b200_'


def segment_name(token: str, rank: int) -> str:
    return f'{NAME_PREFIX}{token}_r{rank}'


class HostSegments:
    """One shared host segment per rank of `group`, all mapped by every rank."""

    def __init__(self, group: dist.ProcessGroup, num_bytes: int):
        if num_bytes <= 0:
            raise ValueError('num_bytes must be positive')
        _C = require_ext()
        self.group, self.rank, self.num_ranks = group, group.rank(), group.size()
        self.num_bytes = int(num_bytes)
        token = [secrets.token_hex(6) if self.rank == 0 else None]
        dist.broadcast_object_list(token, src=dist.get_global_rank(group, 0), group=group)
        own = _C.HostSegment(segment_name(token[0], self.rank), self.num_bytes, True)
        names: List[Optional[str]] = [None] * self.num_ranks
        dist.all_gather_object(names, own.name(), group)  # every segment exists once this returns
        self._segs = [own if r == self.rank else _C.HostSegment(names[r], self.num_bytes, False)
                      for r in range(self.num_ranks)]
        dist.barrier(group)
        self._ptrs: Optional[List[int]] = None

    @property
    def names(self) -> List[str]:
        return [s.name() for s in self._segs]

    def view(self, rank: int) -> torch.Tensor:
        """CPU uint8 tensor over `rank`'s segment (shares the memory)."""
        return self._segs[rank].host_view(0, self.num_bytes)

    def device_ptrs(self) -> List[int]:
        """Device addresses of every rank's segment (registered with CUDA on first use)."""
        if self._ptrs is None:
            self._ptrs = [s.device_ptr() for s in self._segs]
        return self._ptrs

    def destroy(self) -> None:
        """Collective: the ranks meet before any segment is unmapped or unlinked."""
        if self._segs:
            dist.barrier(self.group)
            for s in self._segs:
                s.destroy()
            self._segs = []
            self._ptrs = None


def fetch_rows_reference(indices: torch.Tensor, views: List[torch.Tensor], entries_per_rank: int,
                         hidden: int) -> torch.Tensor:
    """Torch restatement of the Engram fetch from host segments: row (i % entries) of rank
    i // entries, bf16; an index outside [0, ranks * entries) gives a zero row."""
    idx = indices.long().cpu()
    out = torch.zeros((idx.numel(), hidden), dtype=torch.bfloat16)
    total = entries_per_rank * len(views)
    for t, i in enumerate(idx.tolist()):
        if 0 <= i < total:
            r, e = divmod(i, entries_per_rank)
            out[t] = views[r][e * hidden * 2:(e + 1) * hidden * 2].view(torch.bfloat16)
    return out
