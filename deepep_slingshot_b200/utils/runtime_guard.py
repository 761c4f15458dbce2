"""Guard against two NCCL runtimes in one process.

torch.distributed's NCCL backend runs on the `libnccl.so` that PyTorch was linked against (in a
wheel install: the `nvidia-nccl` package's `lib/libnccl.so.2`). If another library maps a second,
different `libnccl.so` (a system copy of another version, say), the two runtimes keep separate
communicator state and NVLS/IPC resources; this fails later in ways that are hard to trace. The
reference's package checks the same at import (`check_nccl_so`, deep_ep/__init__.py, as patched by
patches/deepep-bd1e1669-cxi-full.patch:13-30, tested by backend/tests/test_nccl_runtime_guard.py):

  * only mapped files whose name is `libnccl.so[.N...]` are runtimes; network, tuner and GIN
    plugins (`libnccl-net.so`, `libnccl-tuner*.so`, ...) are not;
  * one runtime mapped several times is fine; two different files are an error unless their
    contents are identical (the same library reached through two paths);
  * when the expected runtime is known, a different mapped runtime is an error.

Unlike the reference, a process with no mapped runtime passes: PyTorch builds may link NCCL
statically, and this library itself moves data through CUDA IPC, not NCCL.
`DEEPEP_B200_SUPPRESS_NCCL_CHECK=1` skips the check.
"""
import filecmp
import glob
import os
import re
from typing import List, Optional

_RUNTIME_NAME = re.compile(r'libnccl\.so(?:\.\d+)*')


class NcclRuntimeError(RuntimeError):
    """Two NCCL runtimes, or an unexpected one, are mapped into this process."""
    pass


def mapped_nccl_runtimes(maps_text: Optional[str] = None) -> List[str]:
    """Paths of the NCCL runtimes mapped into this process, in first-mapped order, without repeats.
    `maps_text` is the content of `/proc/self/maps` (read when None)."""
    if maps_text is None:
        try:
            with open('/proc/self/maps') as f:
                maps_text = f.read()
        except OSError:
            return []
    seen: List[str] = []
    for line in maps_text.splitlines():
        fields = line.split(maxsplit=5)
        if len(fields) < 6:
            continue
        path = fields[5].strip()
        if path.endswith(' (deleted)'):
            path = path[:-len(' (deleted)')]
        if _RUNTIME_NAME.fullmatch(os.path.basename(path)) and path not in seen:
            seen.append(path)
    return seen


def expected_nccl_runtime() -> Optional[str]:
    """The runtime PyTorch's wheel ships (`nvidia/nccl/lib/libnccl.so*`), or None if there is none."""
    try:
        import nvidia.nccl as pkg
    except ImportError:
        return None
    for root in getattr(pkg, '__path__', []):
        found = sorted(glob.glob(os.path.join(root, 'lib', 'libnccl.so*')))
        if found:
            return found[0]
    return None


def _same_library(a: str, b: str) -> bool:
    if a == b:
        return True
    try:
        return os.path.samefile(a, b) or filecmp.cmp(a, b, shallow=False)
    except OSError:
        return False


def check_nccl_runtime(maps_text: Optional[str] = None, expected: Optional[str] = '') -> Optional[str]:
    """Raise `NcclRuntimeError` if two different NCCL runtimes are mapped, or if the mapped runtime
    is not `expected` (default: `expected_nccl_runtime()`; None disables that part). Returns the
    mapped runtime's path (None when no runtime is mapped)."""
    if os.environ.get('DEEPEP_B200_SUPPRESS_NCCL_CHECK', '0') == '1':
        return None
    runtimes = mapped_nccl_runtimes(maps_text)
    if not runtimes:
        return None
    first = runtimes[0]
    for other in runtimes[1:]:
        if not _same_library(first, other):
            raise NcclRuntimeError(f'two NCCL runtimes are mapped into this process: {first} and {other} '
                                   '(set DEEPEP_B200_SUPPRESS_NCCL_CHECK=1 to skip this check)')
    if expected == '':
        expected = expected_nccl_runtime()
    if expected is not None and not _same_library(first, expected):
        raise NcclRuntimeError(f'the mapped NCCL runtime {first} is not the one PyTorch ships ({expected}) '
                               '(set DEEPEP_B200_SUPPRESS_NCCL_CHECK=1 to skip this check)')
    return first
