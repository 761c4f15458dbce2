"""Analysis of multi-rank device timelines written by `harness.trace_capture` (Chrome-trace JSON).

    python -m deepep_slingshot_b200.harness.analyze_trace trace_ep8/trace.json

For every traced step it reports, per phase (stage, notify, pull, combine, ...):
  * start / end spread over ranks (inter-rank skew: how long the earliest rank waits for the last);
  * busy time = union of the phase's block intervals on each rank (no double counting), and
    duty = busy / window (how much of the phase window the GPU actually worked on it);
and the step's critical path: the chain of the latest-ending rank per phase, with the idle gaps
between phases (host launch gaps show up there). The reference's campaign tooling computes the same
kinds of quantities (non-double-counted unions, receiver duty: backend/tools/analyze_profiles.py,
harness/pipeline_1102/receiver_duty.py).
"""
import json
import sys
from collections import defaultdict
from typing import Dict, List, Tuple

PHASE_ORDER = ['dispatch.wait_receivers', 'dispatch.count', 'dispatch.count.exchange', 'dispatch.stage',
               'dispatch.pull', 'combine.push_warp', 'combine.block', 'll_dispatch.send', 'll_dispatch.recv',
               'll_combine.send', 'll_combine.recv', 'barrier', 'pp.copy']


def _union(intervals: List[Tuple[float, float]]) -> float:
    total, cur = 0.0, None
    for s, e in sorted(intervals):
        if cur is None or s > cur[1]:
            if cur is not None:
                total += cur[1] - cur[0]
            cur = [s, e]
        else:
            cur[1] = max(cur[1], e)
    if cur is not None:
        total += cur[1] - cur[0]
    return total


def split_steps(events: List[dict], gap_us: float = 50.0) -> List[List[dict]]:
    """Split one rank's events into steps at gaps between dispatch starts (the count kernel's first
    record of a step)."""
    events = sorted(events, key=lambda e: e['ts'])
    starts = sorted(e['ts'] for e in events if e['name'] == 'dispatch.wait_receivers')
    bounds = [t for i, t in enumerate(starts) if i == 0 or t - starts[i - 1] > gap_us]
    if not bounds:
        return [events]
    steps: List[List[dict]] = [[] for _ in bounds]
    for e in events:
        idx = max(0, sum(1 for b in bounds if b <= e['ts'] + 1e-6) - 1)
        steps[idx].append(e)
    return steps


def analyze(trace: dict) -> List[dict]:
    """Per-step phase rows (window, busy union, duty, skew over ranks) of a Chrome trace written by
    `harness.trace_capture`."""
    by_rank: Dict[int, List[dict]] = defaultdict(list)
    for e in trace['traceEvents']:
        by_rank[e['pid']].append(e)
    per_rank_steps = {r: split_steps(ev) for r, ev in by_rank.items()}
    n_steps = min(len(s) for s in per_rank_steps.values())
    report = []
    for s in range(n_steps):
        phases = {}
        for name in PHASE_ORDER:
            rows = []
            for r, steps in per_rank_steps.items():
                iv = [(e['ts'], e['ts'] + e['dur']) for e in steps[s] if e['name'] == name]
                if iv:
                    lo, hi = min(a for a, _ in iv), max(b for _, b in iv)
                    rows.append({'rank': r, 'start': lo, 'end': hi, 'busy': _union(iv)})
            if rows:
                phases[name] = {
                    'start_spread_us': max(x['start'] for x in rows) - min(x['start'] for x in rows),
                    'end_spread_us': max(x['end'] for x in rows) - min(x['end'] for x in rows),
                    'window_us': max(x['end'] for x in rows) - min(x['start'] for x in rows),
                    'duty': min(1.0, sum(x['busy'] for x in rows) /
                                max(1e-9, sum(x['end'] - x['start'] for x in rows))),
                    'last_rank': max(rows, key=lambda x: x['end'])['rank'],
                    'end': max(x['end'] for x in rows), 'start': min(x['start'] for x in rows)}
        chain, prev_end = [], None
        # The stage runs concurrently with the pull (stage warps of the pull launch), so the chain is
        # count -> pull -> combine; the stage's own window is reported among the phases.
        for name in ('dispatch.count', 'dispatch.pull', 'combine.block'):
            if name in phases:
                p = phases[name]
                gap = 0.0 if prev_end is None else max(0.0, p['start'] - prev_end)
                chain.append({'phase': name, 'gap_before_us': gap, 'span_us': p['end'] - max(p['start'], prev_end or p['start'])})
                prev_end = p['end']
        report.append({'step': s, 'phases': phases, 'critical_path': chain})
    return report


def main(argv=None):
    argv = argv if argv is not None else sys.argv[1:]
    with open(argv[0] if argv else 'trace_out/trace.json') as f:
        rep = analyze(json.load(f))
    for st in rep:
        print(f"--- step {st['step']}")
        for name, p in st['phases'].items():
            print(f"{name:32s} window {p['window_us']:8.1f} us  start spread {p['start_spread_us']:7.1f}  "
                  f"end spread {p['end_spread_us']:7.1f}  duty {p['duty']:.2f}  last rank {p['last_rank']}")
        print('critical path: ' + ' -> '.join(f"{c['phase']} (+{c['gap_before_us']:.0f} gap, {c['span_us']:.0f} us)"
                                              for c in st['critical_path']))


if __name__ == '__main__':
    main()
