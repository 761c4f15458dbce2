"""Symmetric side regions for the elastic API's experimental features (pipeline send/recv, AGRS
all-gather sessions, Engram storage), and a CPU/gloo oracle of the same semantics.

`SymmetricRegion(group, data_bytes)` allocates one CUDA-IPC region per rank ([64 KiB control | data]),
exchanges the handles over `torch.distributed` and opens every peer's region. Construction is a
collective call. The reference carves the same features out of its NCCL symmetric window
([DE]csrc/elastic/buffer.hpp:212-470); here each feature owns a region so they never alias.
"""
from typing import Callable, Optional, Tuple

import torch
import torch.distributed as dist

from .._ext import require_ext
from ..utils import lifecycle


def _default_timeout() -> float:
    import os
    return float(os.environ.get('DEEPEP_B200_GPU_TIMEOUT_SECS', '100'))


class SymmetricRegion:
    """One CUDA-IPC region per rank of `group` with `data_bytes` of payload (collective)."""

    def __init__(self, group: dist.ProcessGroup, data_bytes: int, timeout_secs: Optional[float] = None):
        _C = require_ext()
        used_before = lifecycle.snapshot()
        self.group = group
        self.rank = group.rank()
        self.num_ranks = group.size()
        self.runtime = _C.SymmetricRegion(self.rank, self.num_ranks, int(data_bytes),
                                          _default_timeout() if timeout_secs is None else float(timeout_secs))
        handles = [None] * self.num_ranks
        dist.all_gather_object(handles, bytes(self.runtime.get_local_ipc_handle()), group)
        self.runtime.sync(handles)
        torch.cuda.synchronize()
        dist.barrier(group)
        lifecycle.record('create', 'SymmetricRegion', self, int(data_bytes), used_before)

    @property
    def data_bytes(self) -> int:
        return self.runtime.data_bytes()

    def destroy(self) -> None:
        if self.runtime is not None:
            self.runtime.destroy()
            self.runtime = None
            lifecycle.record('destroy', 'SymmetricRegion', self)

    def check_error(self) -> None:
        self.runtime.check_error()

    def barrier(self) -> None:
        self.runtime.barrier()


def ring_neighbours(rank: int, num_ranks: int) -> Tuple[int, int]:
    """(prev, next) rank of the pipeline ring."""
    return (rank + num_ranks - 1) % num_ranks, (rank + 1) % num_ranks


class ReferenceSideFeatures:
    """CPU/gloo oracle of pipeline send/recv, AGRS all-gather and Engram fetch (torch.distributed
    point-to-point and all_gather). Mirrors the call shapes of the GPU implementation."""

    def __init__(self, group: dist.ProcessGroup):
        self.group = group
        self.rank = group.rank()
        self.num_ranks = group.size()
        self._storage: Optional[torch.Tensor] = None
        self._entries = 0

    # pipeline
    def pp_send(self, t: torch.Tensor, dst_rank_idx: int) -> None:
        prev, nxt = ring_neighbours(self.rank, self.num_ranks)
        assert dst_rank_idx in (prev, nxt)
        dist.send(t.contiguous(), dist.get_global_rank(self.group, dst_rank_idx), group=self.group)

    def pp_recv(self, t: torch.Tensor, src_rank_idx: int) -> None:
        prev, nxt = ring_neighbours(self.rank, self.num_ranks)
        assert src_rank_idx in (prev, nxt)
        dist.recv(t, dist.get_global_rank(self.group, src_rank_idx), group=self.group)

    # AGRS
    def all_gather(self, t: torch.Tensor) -> torch.Tensor:
        out = [torch.empty_like(t) for _ in range(self.num_ranks)]
        dist.all_gather(out, t.contiguous(), group=self.group)
        return torch.stack(out)

    # Engram
    def engram_write(self, storage: torch.Tensor) -> None:
        parts = [torch.empty_like(storage) for _ in range(self.num_ranks)]
        dist.all_gather(parts, storage.contiguous(), group=self.group)
        self._storage = torch.cat(parts)
        self._entries = storage.shape[0]

    def engram_fetch(self, indices: torch.Tensor) -> Callable[[], torch.Tensor]:
        assert self._storage is not None, 'call engram_write first'
        idx = indices.long()
        valid = (idx >= 0) & (idx < self._storage.shape[0])
        out = torch.zeros((idx.numel(), self._storage.shape[1]), dtype=self._storage.dtype)
        out[valid] = self._storage[idx[valid]]
        return lambda: out
