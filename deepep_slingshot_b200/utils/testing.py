"""Timing helpers: CUDA-event benchmark with an L2 flush, per-kernel timing through the torch
profiler, and rank-max aggregation (the reference's `bench` / `bench_kineto`,
[DE]deep_ep/utils/testing.py:60-219, re-written for this library)."""
import os
import sys
from typing import Callable, Dict, List, Optional, Sequence, Tuple, Union

import torch
import torch.distributed as dist

_L2_FLUSH_BYTES = 256 << 20  # larger than the B200's 126 MB L2


def _flush_buffer() -> torch.Tensor:
    buf = getattr(_flush_buffer, '_buf', None)
    if buf is None or buf.device.index != torch.cuda.current_device():
        buf = torch.empty(_L2_FLUSH_BYTES, dtype=torch.uint8, device='cuda')
        _flush_buffer._buf = buf
    return buf


def bench(fn: Callable[[], object], num_warmups: int = 5, num_tests: int = 20, flush_l2: bool = True,
          post_fn: Optional[Callable[[], object]] = None) -> Tuple[float, float, float, List[float]]:
    """Time `fn` with CUDA events on the current stream: warm-ups, then `num_tests` timed calls,
    each after an L2-evicting write when `flush_l2`. Returns (mean, min, max, all) in seconds; the
    first timed sample is dropped from the statistics (it often carries allocator growth)."""
    for _ in range(num_warmups):
        fn()
        if post_fn is not None:
            post_fn()
    torch.cuda.synchronize()
    flush = _flush_buffer() if flush_l2 else None
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(num_tests)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(num_tests)]
    for i in range(num_tests):
        if flush is not None:
            flush.zero_()
        starts[i].record()
        fn()
        ends[i].record()
        if post_fn is not None:
            post_fn()
    torch.cuda.synchronize()
    times = [s.elapsed_time(e) / 1e3 for s, e in zip(starts, ends)]
    stats = times[1:] if len(times) > 1 else times
    return sum(stats) / len(stats), min(stats), max(stats), times


def rank_max(values: Sequence[float], group: Optional[dist.ProcessGroup] = None) -> List[float]:
    """Element-wise max over the ranks of `group` (per-iteration rank-max times)."""
    t = torch.tensor(list(values), dtype=torch.float64, device='cuda')
    if dist.is_initialized() and (group is None or group.size() > 1):
        dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return t.tolist()


def bench_kineto(fn: Callable[[], object], kernel_names: Union[str, Sequence[str]], num_tests: int = 30,
                 flush_l2: bool = True, barrier_group: Optional[dist.ProcessGroup] = None,
                 suppress_kineto_output: bool = True) -> Union[float, List[float]]:
    """Mean device seconds per call of each kernel whose name contains one of `kernel_names`,
    from the torch profiler's CUDA activity (kernels only, so host gaps do not count). With
    `barrier_group` the ranks are aligned by a barrier before the profiled calls."""
    single = isinstance(kernel_names, str)
    names = [kernel_names] if single else list(kernel_names)
    flush = _flush_buffer() if flush_l2 else None
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    if barrier_group is not None:
        dist.barrier(barrier_group)
    acts = [torch.profiler.ProfilerActivity.CUDA]
    with torch.profiler.profile(activities=acts) as prof:
        for _ in range(num_tests):
            if flush is not None:
                flush.zero_()
            fn()
        torch.cuda.synchronize()
    totals: Dict[str, float] = {n: 0.0 for n in names}
    counts: Dict[str, int] = {n: 0 for n in names}
    for evt in prof.events():
        if evt.device_type != torch.autograd.DeviceType.CUDA:
            continue
        for n in names:
            if n in evt.name:
                totals[n] += evt.device_time_total if hasattr(evt, 'device_time_total') else evt.cuda_time_total
                counts[n] += 1
    out = [totals[n] / 1e6 / num_tests if counts[n] else 0.0 for n in names]
    return out[0] if single else out


def hash_tensor(t: torch.Tensor) -> str:
    """SHA-256 of a tensor's bytes (inputs / routes in benchmark records)."""
    import hashlib
    return hashlib.sha256(t.detach().contiguous().cpu().view(torch.uint8).numpy().tobytes()).hexdigest()


def flush_l2_cache(enabled: bool = True) -> None:
    """Evict the GPU L2 (126 MB on B200) with a 256 MB write."""
    if enabled:
        _flush_buffer().zero_()


class empty_suppress:
    """No-op context manager (the counterpart of `suppress_stdout_stderr`)."""

    def __enter__(self):
        return self

    def __exit__(self, *_):
        return False


class suppress_stdout_stderr:
    """Silence the process's stdout/stderr file descriptors (also output of C/C++ code) inside the block."""

    def __enter__(self):
        sys.stdout.flush()
        sys.stderr.flush()
        self._devnull = os.open(os.devnull, os.O_WRONLY)
        self._saved = [os.dup(1), os.dup(2)]
        os.dup2(self._devnull, 1)
        os.dup2(self._devnull, 2)
        return self

    def __exit__(self, *_):
        sys.stdout.flush()
        sys.stderr.flush()
        os.dup2(self._saved[0], 1)
        os.dup2(self._saved[1], 2)
        for fd in self._saved + [self._devnull]:
            os.close(fd)
        return False
