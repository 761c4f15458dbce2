"""Lifecycle records of communication buffers, for leak audits over create/destroy cycles.

With `DEEPEP_B200_LIFECYCLE_LOG=<path>` set (`{rank}` in the path is replaced by the global rank),
`Buffer`, `ElasticBuffer` and `SymmetricRegion` append one JSON line per construction and per
destruction: the kind and id of the object, the bytes it requested, how many objects of that kind
are alive, and the device memory in use (`total - free` from the driver, measured after a
synchronize, a garbage collection and `torch.cuda.empty_cache()`, so that only memory held outside
PyTorch's cache counts; logging therefore changes allocator behaviour and is a diagnostic mode).
`harness.analyze_lifecycle` audits such a log. The reference audits its NIC context pools the same
way (backend/tools/analyze_lifecycle.py, tested by backend/tests/test_lifecycle_analysis.py): every
cycle must reuse or release what it took, and physical usage must not grow from cycle to cycle.
"""
import gc
import json
import os
import threading
import time
from collections import Counter
from typing import Optional, Tuple

_ENV = 'DEEPEP_B200_LIFECYCLE_LOG'
_lock = threading.Lock()
_alive: Counter = Counter()


def enabled() -> bool:
    """Whether lifecycle logging is on (`DEEPEP_B200_LIFECYCLE_LOG` set)."""
    return bool(os.environ.get(_ENV))


def _log_path() -> Tuple[str, int]:
    rank = 0
    try:
        import torch.distributed as dist
        if dist.is_available() and dist.is_initialized():
            rank = dist.get_rank()
    except Exception:
        pass
    return os.environ[_ENV].replace('{rank}', str(rank)), rank


def device_used_bytes() -> int:
    """Device memory in use outside PyTorch's cache (driver view)."""
    import torch
    torch.cuda.synchronize()
    gc.collect()
    torch.cuda.empty_cache()
    free, total = torch.cuda.mem_get_info()
    return int(total - free)


def snapshot() -> Optional[int]:
    """Device memory in use before a construction (None unless logging is on); passed to `record`
    as `used_before` so the audit can compare what an object took with what it requested."""
    return device_used_bytes() if enabled() else None


def record(phase: str, kind: str, obj: object, requested_bytes: int = 0, used_before: Optional[int] = None,
           extra: Optional[dict] = None) -> None:
    """Append a lifecycle record (`phase` is 'create' or 'destroy'); a no-op unless logging is on."""
    if not enabled():
        return
    with _lock:
        if phase == 'create':
            _alive[kind] += 1
        elif phase == 'destroy':
            _alive[kind] -= 1
        alive = _alive[kind]
    path, rank = _log_path()
    rec = {'phase': phase, 'kind': kind, 'id': id(obj), 'rank': rank, 'requested_bytes': int(requested_bytes),
           'alive': alive, 'device_used_bytes': device_used_bytes(), 'time': time.time()}
    if used_before is not None:
        rec['used_before_bytes'] = int(used_before)
    if extra:
        rec.update(extra)
    with _lock:
        with open(path, 'a') as f:
            f.write(json.dumps(rec) + '\n')
