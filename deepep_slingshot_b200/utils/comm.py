"""NCCL communicator handles of process groups: interface parity with the reference's
`deep_ep.utils.comm` (`NCCLCommHandle`, `get_nccl_comm_handle`, `destroy_all_managed_nccl_comm`).

The reference hands its NCCL communicator to its GIN transport, creating one of its own when the
installed PyTorch cannot expose the process group's. This library's transport is CUDA IPC over
NVLink, so it never needs, and never creates, a communicator: the torch process group is the
communicator. These helpers only expose the process group's own NCCL communicator (through
PyTorch's `_comm_ptr()` on the NCCL backend) to callers that want the raw pointer, e.g. to share it
with another NCCL-based library; every handle is therefore unmanaged, and nothing is destroyed here.
"""
from typing import Dict

import torch
import torch.distributed as dist


class NCCLCommHandle:
    """The raw NCCL communicator (`ncclComm_t` as an integer) of a process group."""

    def __init__(self, nccl_comm: int, managed: bool = False) -> None:
        if managed:
            raise ValueError('this library never creates NCCL communicators, so it manages none')
        self.nccl_comm = int(nccl_comm)
        self.managed = False

    def get(self) -> int:
        return self.nccl_comm


_HANDLES: Dict[int, NCCLCommHandle] = {}


def get_nccl_comm_handle(group: dist.ProcessGroup) -> NCCLCommHandle:
    """Handle of `group`'s NCCL communicator, cached per group. Raises RuntimeError when the group
    has no NCCL backend on CUDA or the installed PyTorch does not expose the communicator."""
    key = id(group)
    if key in _HANDLES:
        return _HANDLES[key]
    try:
        backend = group._get_backend(torch.device('cuda'))
    except Exception as exc:  # no CUDA backend registered for this group (e.g. gloo only)
        raise RuntimeError(f'the process group has no CUDA (NCCL) backend: {exc}') from exc
    comm_ptr = getattr(backend, '_comm_ptr', None)
    if comm_ptr is None:
        raise RuntimeError('this PyTorch does not expose the NCCL communicator of a process group '
                           '(ProcessGroupNCCL._comm_ptr); the library itself does not need it')
    _HANDLES[key] = NCCLCommHandle(comm_ptr())
    return _HANDLES[key]


def destroy_all_managed_nccl_comm() -> None:
    """Drop every cached handle. No communicator is destroyed: the process groups own theirs."""
    _HANDLES.clear()
