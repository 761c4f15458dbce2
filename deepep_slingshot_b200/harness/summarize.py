"""Summaries of `ep_benchmark` records: `summary.csv` (per case and op: median / p95 / mean of the
per-iteration rank-max time, GB/s, worst host time per iteration) and `repeatability.json` (spread
of the median over seeds). The reference's summarizer computes the same quantities
(backend/tests/summarize.py:11-59).

    python -m deepep_slingshot_b200.harness.summarize ep_results
"""
import csv
import glob
import json
import os
import statistics
import sys
from collections import defaultdict
from typing import Dict, List

CASE_KEYS = ('model', 'tokens_per_rank', 'ranks', 'dispatch_dtype', 'routing', 'seed', 'op')


def _pct(values: List[float], q: float) -> float:
    s = sorted(values)
    if not s:
        return float('nan')
    k = min(len(s) - 1, max(0, int(round(q * (len(s) - 1)))))
    return s[k]


def load_timings(out_dir: str) -> Dict[tuple, List[dict]]:
    """Timing records of every rank grouped by (case, op)."""
    groups: Dict[tuple, List[dict]] = defaultdict(list)
    for path in sorted(glob.glob(os.path.join(out_dir, 'timings-rank*.jsonl'))):
        with open(path) as f:
            for line in f:
                rec = json.loads(line)
                if rec.get('kind') == 'timing':
                    groups[tuple(rec[k] for k in CASE_KEYS)].append(rec)
    return groups


def summarize_dir(out_dir: str) -> List[dict]:
    """Write `summary.csv` and `repeatability.json` for a results directory; returns the rows."""
    rows = []
    for key, recs in load_timings(out_dir).items():
        rmax = recs[0]['rank_max_us']
        med = statistics.median(rmax)
        total_bytes = sum(r['bytes'] for r in recs)
        worst_bytes = max(r['bytes'] for r in recs)
        row = dict(zip(CASE_KEYS, key))
        row.update({
            'median_rank_max_us': round(med, 2), 'p95_rank_max_us': round(_pct(rmax, 0.95), 2),
            'mean_rank_max_us': round(statistics.fmean(rmax), 2), 'min_rank_max_us': round(min(rmax), 2),
            'gbps_per_rank': round(total_bytes / len(recs) / (med * 1e-6) / 1e9, 1),
            'gbps_bottleneck_rank': round(worst_bytes / (med * 1e-6) / 1e9, 1),
            'max_host_us_per_iteration': round(max(r['max_host_us_per_iteration'] for r in recs), 1),
            'ranks_reporting': len(recs)})
        rows.append(row)
    rows.sort(key=lambda r: tuple(str(r[k]) for k in CASE_KEYS))
    if rows:
        with open(os.path.join(out_dir, 'summary.csv'), 'w', newline='') as f:
            w = csv.DictWriter(f, fieldnames=list(rows[0].keys()))
            w.writeheader()
            w.writerows(rows)
    rep = defaultdict(list)
    for r in rows:
        rep['|'.join(str(r[k]) for k in CASE_KEYS if k != 'seed')].append(r['median_rank_max_us'])
    repeat = {}
    for k, meds in rep.items():
        mean = statistics.fmean(meds)
        repeat[k] = {'medians_us': meds, 'mean_us': round(mean, 2),
                     'cv': round(statistics.pstdev(meds) / mean, 4) if len(meds) > 1 and mean > 0 else 0.0}
    with open(os.path.join(out_dir, 'repeatability.json'), 'w') as f:
        json.dump(repeat, f, indent=1)
    return rows


if __name__ == '__main__':
    for row in summarize_dir(sys.argv[1] if len(sys.argv) > 1 else 'ep_results'):
        print(row)
