"""Locate the NVIDIA runtime packages a process uses (NCCL, NVSHMEM): interface parity with the
reference's `deep_ep.utils.find_pkgs` (`find_pkg_root`, `find_nccl_root`, `find_nvshmem_root`),
which its build and import-time NCCL check call.

This library needs neither at build time (it compiles against CUDA only and moves data through
CUDA IPC), so here the helpers serve diagnostics: which NCCL install the process would load (the
runtime guard compares it with what is mapped) and whether an NVSHMEM install is present.

Search order for package `name`:
  1. the environment: `DEEPEP_B200_<NAME>_ROOT_DIR`, then `<NAME>_DIR`;
  2. installed Python distributions named `nvidia-<name>...` (the pip wheels, e.g.
     `nvidia-nccl-cu12`), in `sys.path` order, the first whose files contain `lib_name` (its
     root is the directory above that file's `lib/`), or with an `nvidia/<name>` directory.
"""
import functools
import os
import sys
from importlib import metadata
from typing import Iterable, Optional


def _dist_root(dist, name: str, lib_name: Optional[str]) -> Optional[str]:
    site = os.path.dirname(str(getattr(dist, '_path', '') or ''))
    if lib_name is not None:
        for f in dist.files or []:
            if os.path.basename(str(f)).startswith(lib_name):
                lib_dir = os.path.dirname(str(f.locate()))
                return os.path.dirname(lib_dir) if os.path.basename(lib_dir) == 'lib' else lib_dir
        return None
    cand = os.path.join(site, 'nvidia', name)
    return cand if os.path.isdir(cand) else None


def find_pkg_root(name: str, lib_name: Optional[str] = None, optional: bool = False,
                  dists: Optional[Iterable] = None) -> Optional[str]:
    """Root directory of NVIDIA package `name` (see the module docstring for the search order).
    Raises FileNotFoundError when nothing is found, unless `optional` (then None). `dists` replaces
    the installed distributions (tests)."""
    upper = name.upper()
    for var in (f'DEEPEP_B200_{upper}_ROOT_DIR', f'{upper}_DIR'):
        if os.environ.get(var):
            return os.environ[var]
    order = {p: i for i, p in enumerate(sys.path)}
    found, rank = None, None
    for dist in (dists if dists is not None else metadata.distributions()):
        dname = (dist.metadata['Name'] or '').lower().replace('_', '-')
        if not dname.startswith(f'nvidia-{name}'):
            continue
        site = os.path.dirname(str(getattr(dist, '_path', '') or ''))
        r = order.get(site, len(sys.path))
        if rank is not None and r >= rank:
            continue
        root = _dist_root(dist, name, lib_name)
        if root is not None:
            found, rank = root, r
    if found is None and not optional:
        raise FileNotFoundError(f'no installation of NVIDIA package {name!r} found '
                                f'(set DEEPEP_B200_{upper}_ROOT_DIR to point at it)')
    return found


@functools.lru_cache(maxsize=None)
def find_nccl_root(optional: bool = False) -> Optional[str]:
    """Root of the NCCL install (the directory holding `lib/libnccl.so*`)."""
    return find_pkg_root('nccl', 'libnccl.so', optional)


@functools.lru_cache(maxsize=None)
def find_nvshmem_root(optional: bool = True) -> Optional[str]:
    """Root of an NVSHMEM install, if any (this library does not use NVSHMEM)."""
    return find_pkg_root('nvshmem', 'libnvshmem', optional)
