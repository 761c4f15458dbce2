"""Interval analysis of torch.profiler traces written by `harness.profile_capture`.

    python -m deepep_slingshot_b200.harness.analyze_profiles prof_ep8

`profile_capture` marks every profiled call with a `ep/<operation>/iteration<i>` range. For each
operation, rank and iteration this computes, from the Chrome trace's device events:
  * kernel span (first kernel start to last kernel end), kernel union (time with at least one
    kernel running; concurrent kernels are not double counted), gap = span - union (idle device
    time inside the span: launch and synchronisation bubbles), overlap = sum of kernel durations -
    union (time kernels ran concurrently);
  * the union of host synchronisation calls (`cudaDeviceSynchronize`, `cudaStreamSynchronize`,
    `cudaEventSynchronize`);
  * per-kernel totals.
A kernel belongs to the iteration whose range contains its launch call (the runtime call with the
same correlation id); traces without correlation ids fall back to the window from one iteration's
start to the next one's. Results are diagnostic (`status: DIAGNOSTIC_ONLY`): profiled runs are
never benchmark values. The analysis fails (ValueError) on traces without device events, on missing
iterations, on malformed intervals, when a rank's trace or summary is missing, and when the ranks
profiled different cases. The reference's `backend/tools/analyze_profiles.py` (tested by
backend/tests/test_profile_analysis.py:13-85) computes the same span/union/gap/overlap figures.
"""
import glob
import json
import math
import os
import re
import sys
from collections import defaultdict
from typing import Dict, List, Sequence, Tuple

SYNC_CALLS = ('cudaDeviceSynchronize', 'cudaStreamSynchronize', 'cudaEventSynchronize')
_MARK = re.compile(r'ep/(?P<op>[A-Za-z0-9_]+)/iteration(?P<it>\d+)$')
_DEVICE_CATS = ('kernel', 'gpu_memcpy', 'gpu_memset')


def interval_stats(intervals: Sequence[Tuple[float, float]]) -> Dict[str, float]:
    """span / union / gap / overlap / busy (sum of durations) of closed intervals [start, end]."""
    for s, e in intervals:
        if not (math.isfinite(s) and math.isfinite(e)) or e < s:
            raise ValueError(f'invalid interval ({s}, {e})')
    if not intervals:
        return {'span': 0.0, 'union': 0.0, 'gap': 0.0, 'overlap': 0.0, 'busy': 0.0}
    union, cur_s, cur_e = 0.0, None, None
    for s, e in sorted(intervals):
        if cur_e is None or s > cur_e:
            if cur_e is not None:
                union += cur_e - cur_s
            cur_s, cur_e = s, e
        else:
            cur_e = max(cur_e, e)
    union += cur_e - cur_s
    span = max(e for _, e in intervals) - min(s for s, _ in intervals)
    busy = sum(e - s for s, e in intervals)
    return {'span': span, 'union': union, 'gap': span - union, 'overlap': busy - union, 'busy': busy}


def _interval(ev: dict) -> Tuple[float, float]:
    s, d = float(ev.get('ts', float('nan'))), float(ev.get('dur', float('nan')))
    return s, s + d


def analyze_events(events: List[dict], operation: str, iterations: int) -> Tuple[List[dict], List[dict]]:
    """Per-iteration figures and per-kernel totals of one operation's trace events."""
    complete = [e for e in events if e.get('ph') == 'X']
    marks = {}
    for e in complete:
        m = _MARK.match(str(e.get('name', '')))
        if m and m.group('op') == operation and e.get('cat', 'user_annotation') != 'gpu_user_annotation':
            marks.setdefault(int(m.group('it')), e)
    device = [e for e in complete if e.get('cat') in _DEVICE_CATS]
    if not device:
        raise ValueError('No GPU kernel events in the trace (a CPU-only profile)')
    for i in range(iterations):
        if i not in marks:
            raise ValueError(f'{operation}: iteration {i} has no range in the trace')
    order = sorted(marks)
    windows = {}
    for j, i in enumerate(order):
        s, e = _interval(marks[i])
        nxt = _interval(marks[order[j + 1]])[0] if j + 1 < len(order) else float('inf')
        windows[i] = (s, e, nxt)
    # Launch calls (host side) by correlation id.
    launches = {}
    for e in complete:
        corr = (e.get('args') or {}).get('correlation')
        if corr is not None and e.get('cat') in ('cuda_runtime', 'cuda_driver'):
            launches[corr] = e
    per_it: Dict[int, List[dict]] = defaultdict(list)
    for k in device:
        corr = (k.get('args') or {}).get('correlation')
        launch = launches.get(corr)
        for i, (s, e, nxt) in windows.items():
            if launch is not None:
                t = float(launch['ts'])
                if s <= t <= e:
                    per_it[i].append(k)
                    break
            elif s <= float(k['ts']) < nxt:
                per_it[i].append(k)
                break
    syncs = [e for e in complete if e.get('name') in SYNC_CALLS]
    rows, kernels = [], defaultdict(lambda: {'calls': 0, 'total_us': 0.0})
    for i in range(iterations):
        ks = per_it.get(i, [])
        if not ks:
            raise ValueError(f'{operation}: iteration {i} launched no GPU work')
        st = interval_stats([_interval(k) for k in ks])
        s, e, nxt = windows[i]
        end = max(_interval(k)[1] for k in ks)
        sync_iv = [_interval(x) for x in syncs if s <= float(x['ts']) <= max(e, end)]
        rows.append({'operation': operation, 'iteration': i, 'kernels': len(ks),
                     'kernel_span_us': st['span'], 'kernel_union_us': st['union'], 'kernel_gap_us': st['gap'],
                     'kernel_overlap_us': st['overlap'], 'sync_api_union_us': interval_stats(sync_iv)['union']})
        for k in ks:
            kernels[k['name']]['calls'] += 1
            kernels[k['name']]['total_us'] += float(k['dur'])
    krows = [{'operation': operation, 'kernel': n, 'calls': v['calls'], 'total_us': v['total_us'],
              'mean_us': v['total_us'] / v['calls']} for n, v in sorted(kernels.items(), key=lambda x: -x[1]['total_us'])]
    return rows, krows


CASE_KEYS = ('tokens', 'hidden', 'experts', 'topk', 'world', 'dtype')


def analyze(out_dir: str) -> Tuple[dict, List[dict], List[dict]]:
    """Analyze every `<op>-rank<r>-summary.json` / `<op>-rank<r>.json` pair in `out_dir`."""
    summaries = sorted(glob.glob(os.path.join(out_dir, '*-rank*-summary.json')))
    if not summaries:
        raise ValueError(f'no profile summaries in {out_dir}')
    by_op: Dict[str, Dict[int, dict]] = defaultdict(dict)
    for p in summaries:
        with open(p) as f:
            s = json.load(f)
        by_op[s['operation']][int(s['rank'])] = s
    cases = {json.dumps({k: s['case'].get(k) for k in CASE_KEYS}, sort_keys=True)
             for op in by_op.values() for s in op.values()}
    if len(cases) != 1:
        raise ValueError(f'ranks or operations profiled different correctness cases: {sorted(cases)}')
    world = int(json.loads(next(iter(cases)))['world'])
    rows, kernels = [], []
    for op, ranks in sorted(by_op.items()):
        missing = [r for r in range(world) if r not in ranks]
        if missing:
            raise ValueError(f'Missing traces for {op}: ranks {missing}')
        for r in range(world):
            trace = os.path.join(out_dir, f'{op}-rank{r}.json')
            if not os.path.exists(trace):
                raise ValueError(f'Missing traces for {op}: {os.path.basename(trace)}')
            with open(trace) as f:
                events = json.load(f)['traceEvents']
            its = int(ranks[r]['profiled_iterations'])
            rs, ks = analyze_events(events, op, its)
            for x in rs + ks:
                x['rank'] = r
            rows += rs
            kernels += ks
    status = {'status': 'DIAGNOSTIC_ONLY', 'operations': sorted(by_op), 'world': world,
              'case': json.loads(next(iter(cases)))}
    return status, rows, kernels


def main(argv=None) -> int:
    import argparse
    import csv
    p = argparse.ArgumentParser()
    p.add_argument('out_dir')
    args = p.parse_args(argv)
    try:
        status, rows, kernels = analyze(args.out_dir)
    except (OSError, ValueError, KeyError) as e:
        print(f'INVALID: {e}')
        return 1
    for name, data in (('profile_rows.csv', rows), ('profile_kernels.csv', kernels)):
        with open(os.path.join(args.out_dir, name), 'w', newline='') as f:
            wr = csv.DictWriter(f, fieldnames=list(data[0].keys()))
            wr.writeheader()
            wr.writerows(data)
    with open(os.path.join(args.out_dir, 'profile_status.json'), 'w') as f:
        json.dump(status, f, indent=1)
    by_op = defaultdict(list)
    for r in rows:
        by_op[r['operation']].append(r)
    for op, rs in sorted(by_op.items()):
        n = len(rs)
        print(f"{op:16s} span {sum(r['kernel_span_us'] for r in rs) / n:8.1f} us  union "
              f"{sum(r['kernel_union_us'] for r in rs) / n:8.1f}  gap {sum(r['kernel_gap_us'] for r in rs) / n:7.1f}  "
              f"overlap {sum(r['kernel_overlap_us'] for r in rs) / n:7.1f}  (mean over {n} rank-iterations)")
    print(status['status'])
    return 0


if __name__ == '__main__':
    sys.exit(main())
