"""Device trace ring: decode, clock alignment across ranks, Chrome-trace export, validated capture.

The kernels append 40-byte records `[start_ns, end_ns, event, block, smid, rank, a, b]` read from
%globaltimer while tracing is enabled on a `Buffer` (`buffer.enable_trace(capacity)`; a runtime
switch passed to every kernel, no rebuild). The reference keeps the same kind of ring behind a
compile-time pointer (backend/tests/device_trace.cuh:1-29) with host clock ping-pong alignment and an
overflow check that aborts the capture (backend/tests/trace_capture.py:17-69). Here the ranks of one
box share CLOCK_MONOTONIC, so each rank maps its GPU clock onto the host clock with one bracketed
sample (`Buffer.sample_clock`), and an overflowing ring raises instead of returning partial data.
Host calls can be recorded as spans on the same clock (`HostSpans`), which shows how a rank's host
and its kernels interleave. Traced runs are for timelines, never for timing numbers.
"""
import contextlib
import json
import time
from typing import Callable, Dict, List, Optional, Tuple

import numpy as np
import torch
import torch.distributed as dist

TRACE_DTYPE = np.dtype([('start_ns', '<u8'), ('end_ns', '<u8'), ('event', '<i4'), ('block', '<i4'),
                        ('smid', '<i4'), ('rank', '<i4'), ('a', '<i4'), ('b', '<i4')])
assert TRACE_DTYPE.itemsize == 40

# Event ids of `ep::TraceEvent` (csrc/include/ep/abi.h).
TRACE_EVENTS: Dict[int, str] = {
    100: 'dispatch.stage', 101: 'dispatch.wait_receivers', 102: 'dispatch.count',
    103: 'dispatch.count.exchange', 104: 'dispatch.pull',
    110: 'combine.block', 111: 'combine.push_warp',
    120: 'll_dispatch.send', 121: 'll_dispatch.recv', 122: 'll_combine.send', 123: 'll_combine.recv',
    124: 'll_dispatch.recv_gemm',
    130: 'barrier', 140: 'pp.copy',
}


class TraceOverflow(RuntimeError):
    """The device trace ring filled up during a capture (the capture is invalid)."""
    pass


def decode(raw: torch.Tensor) -> np.ndarray:
    """`[n, 40]` uint8 records (as returned by the runtime) -> structured numpy array."""
    return np.frombuffer(raw.contiguous().numpy().tobytes(), dtype=TRACE_DTYPE)


def clock_offset_ns(buffer) -> int:
    """GPU %globaltimer minus host CLOCK_MONOTONIC (ns), from one bracketed sample of this rank."""
    best = None
    for _ in range(5):
        before, gpu, after = buffer.runtime.sample_clock()
        width = after - before
        if best is None or width < best[0]:
            best = (width, gpu - (before + after) // 2)
    return best[1]


def summarize(records: np.ndarray) -> Dict[str, Dict[str, float]]:
    """Per event: count, mean / max duration (µs) and the span of its union on the timeline (µs)."""
    out = {}
    for ev in np.unique(records['event']):
        sel = records[records['event'] == ev]
        dur = (sel['end_ns'] - sel['start_ns']).astype(np.float64) / 1e3
        out[TRACE_EVENTS.get(int(ev), str(int(ev)))] = {
            'count': int(sel.size), 'mean_us': float(dur.mean()), 'max_us': float(dur.max()),
            'union_us': _union_us(sel['start_ns'], sel['end_ns'])}
    return out


def _union_us(starts: np.ndarray, ends: np.ndarray) -> float:
    """Length of the union of [start, end) intervals (non-double-counted busy time)."""
    order = np.argsort(starts)
    total, cur_s, cur_e = 0, None, None
    for s, e in zip(starts[order], ends[order]):
        if cur_e is None or s > cur_e:
            if cur_e is not None:
                total += int(cur_e - cur_s)
            cur_s, cur_e = int(s), int(e)
        else:
            cur_e = max(cur_e, int(e))
    if cur_e is not None:
        total += int(cur_e - cur_s)
    return total / 1e3


class HostSpans:
    """Host-side intervals on CLOCK_MONOTONIC (the clock the device records are aligned to), so the
    calls a rank's host makes appear on the same timeline as its kernels:

        spans = HostSpans()
        with spans.span('host.dispatch_call'):
            buf.dispatch(...)
    """

    def __init__(self) -> None:
        self.spans: List[Tuple[str, int, int]] = []

    @contextlib.contextmanager
    def span(self, name: str):
        start = time.monotonic_ns()
        try:
            yield
        finally:
            self.spans.append((name, start, time.monotonic_ns()))


def to_chrome_trace(records_by_rank: Dict[int, np.ndarray], offsets_ns: Optional[Dict[int, int]] = None,
                    host_by_rank: Optional[Dict[int, List[Tuple[str, int, int]]]] = None) -> dict:
    """Chrome / Perfetto JSON: one process per rank, one thread per (event, block); times on the host
    clock when `offsets_ns` (per-rank GPU-minus-host offsets) are given. `host_by_rank` adds each
    rank's host spans (host clock, thread `host`)."""
    events = []
    t0 = None
    for rank, rec in records_by_rank.items():
        off = (offsets_ns or {}).get(rank, 0)
        for r in rec:
            s = int(r['start_ns']) - off
            t0 = s if t0 is None else min(t0, s)
    for rank, spans in (host_by_rank or {}).items():
        for _, s, _ in spans:
            t0 = s if t0 is None else min(t0, s)
    for rank, spans in (host_by_rank or {}).items():
        for name, s, e in spans:
            events.append({'name': name, 'ph': 'X', 'pid': int(rank), 'tid': 'host', 'ts': (s - (t0 or 0)) / 1e3,
                           'dur': max(e - s, 0) / 1e3, 'args': {}})
    for rank, rec in records_by_rank.items():
        off = (offsets_ns or {}).get(rank, 0)
        for r in rec:
            name = TRACE_EVENTS.get(int(r['event']), str(int(r['event'])))
            s = int(r['start_ns']) - off - (t0 or 0)
            events.append({'name': name, 'ph': 'X', 'pid': int(rank), 'tid': f"{name}/{int(r['block'])}",
                           'ts': s / 1e3, 'dur': max(int(r['end_ns']) - int(r['start_ns']), 0) / 1e3,
                           'args': {'smid': int(r['smid']), 'a': int(r['a']), 'b': int(r['b'])}})
    return {'traceEvents': events, 'displayTimeUnit': 'ns'}


def capture(buffer, fn: Callable[[], None], iterations: int = 1, capacity: int = 1 << 20,
            group: Optional[dist.ProcessGroup] = None, check: Optional[Callable[[], None]] = None):
    """Run `fn` `iterations` times with tracing on; `check` (if given) re-validates results on the
    traced iterations. Returns (records of this rank, GPU-minus-host clock offset). Every rank of
    `group` must call it. Raises `TraceOverflow` when the ring was too small."""
    buffer.runtime.enable_trace(capacity)
    try:
        offset = clock_offset_ns(buffer)
        for _ in range(iterations):
            fn()
            if check is not None:
                check()
        torch.cuda.synchronize()
        raw, appended = buffer.runtime.read_trace(True)
    finally:
        buffer.runtime.disable_trace()
    if appended > capacity:
        raise TraceOverflow(f'trace ring overflow: {appended} records for capacity {capacity}')
    if group is not None:
        dist.barrier(group)
    return decode(raw), offset


def gather_and_write(records: np.ndarray, offset_ns: int, path: Optional[str], group: dist.ProcessGroup,
                     host_spans: Optional[HostSpans] = None) -> dict:
    """All ranks: gather records, offsets and host spans to every rank; rank 0 writes the Chrome
    trace to `path`."""
    world = group.size()
    objs: List = [None] * world
    spans = host_spans.spans if host_spans is not None else []
    dist.all_gather_object(objs, (group.rank(), records.tobytes(), int(offset_ns), spans), group)
    by_rank = {r: np.frombuffer(b, dtype=TRACE_DTYPE) for r, b, _, _ in objs}
    offsets = {r: o for r, _, o, _ in objs}
    host = {r: sp for r, _, _, sp in objs if sp}
    trace = to_chrome_trace(by_rank, offsets, host or None)
    if path and group.rank() == 0:
        with open(path, 'w') as f:
            json.dump(trace, f)
    return trace
