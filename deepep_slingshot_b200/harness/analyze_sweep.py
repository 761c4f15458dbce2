"""Size-sweep fit and bottleneck-rank histogram over an `ep_benchmark` results directory.

    python -m deepep_slingshot_b200.harness.analyze_sweep <results dir> [--json out.json]

The reference's campaign analysis fits its size sweeps and tallies which rank was the slowest
(harness/pipeline_1102: size-sweep fit, rank histograms, effective rate). Here, from the per-rank
timing records (`timings-rank*.jsonl`):
  * per (model, dtype, routing, op), a least-squares fit of the median rank-max time against the
    rank's bytes over the token counts of the sweep, `t = latency + bytes / bandwidth`: the fixed
    cost of one call (launches, flags) and the asymptotic bandwidth, with R^2;
  * per case and op, how often each rank was the slowest over the timed iterations (the rank that
    sets the step time), and the effective rate of the bottleneck rank (its bytes over the median).
"""
import argparse
import json
import statistics
from collections import Counter, defaultdict
from typing import Dict, List, Tuple

from .summarize import CASE_KEYS, load_timings


def fit_line(xs: List[float], ys: List[float]) -> Tuple[float, float, float]:
    """Least squares y = a + b x; returns (a, b, R^2). Needs two distinct x values."""
    n = len(xs)
    mx, my = sum(xs) / n, sum(ys) / n
    sxx = sum((x - mx) ** 2 for x in xs)
    if sxx == 0:
        raise ValueError('a fit needs at least two distinct sizes')
    b = sum((x - mx) * (y - my) for x, y in zip(xs, ys)) / sxx
    a = my - b * mx
    ss_tot = sum((y - my) ** 2 for y in ys)
    ss_res = sum((y - (a + b * x)) ** 2 for x, y in zip(xs, ys))
    return a, b, (1.0 - ss_res / ss_tot) if ss_tot > 0 else 1.0


def sweep_fits(groups: Dict[tuple, List[dict]]) -> List[dict]:
    """One fit per (model, dtype, routing, op) over its token counts (seeds averaged)."""
    idx = {k: i for i, k in enumerate(CASE_KEYS)}
    points: Dict[tuple, Dict[int, List[Tuple[float, float]]]] = defaultdict(lambda: defaultdict(list))
    for key, recs in groups.items():
        med_us = statistics.median(recs[0]['rank_max_us'])
        nbytes = max(r['bytes'] for r in recs)  # the bottleneck rank's bytes
        fam = (key[idx['model']], key[idx['dispatch_dtype']], key[idx['routing']], key[idx['op']])
        points[fam][int(key[idx['tokens_per_rank']])].append((float(nbytes), med_us))
    out = []
    for fam, by_tokens in sorted(points.items()):
        xs, ys = [], []
        for tok in sorted(by_tokens):
            pts = by_tokens[tok]
            xs.append(sum(p[0] for p in pts) / len(pts))
            ys.append(sum(p[1] for p in pts) / len(pts))
        row = dict(zip(('model', 'dispatch_dtype', 'routing', 'op'), fam))
        row['tokens'] = sorted(by_tokens)
        if len(set(xs)) >= 2:
            a, b, r2 = fit_line(xs, ys)
            row.update({'latency_us': round(a, 2), 'bandwidth_gbps': round(1e-3 / b, 1) if b > 0 else None,
                        'r2': round(r2, 4)})
        else:
            row.update({'latency_us': None, 'bandwidth_gbps': None, 'r2': None})
        out.append(row)
    return out


def bottleneck_ranks(groups: Dict[tuple, List[dict]]) -> List[dict]:
    """Per case and op: how often each rank had the largest time of an iteration, and the
    bottleneck rank's effective rate (its bytes over the median rank-max time)."""
    idx = {k: i for i, k in enumerate(CASE_KEYS)}
    out = []
    for key, recs in sorted(groups.items(), key=lambda kv: tuple(str(x) for x in kv[0])):
        # records carry their rank; older ones are in rank order (one file per rank, read in order)
        by_rank = {r.get('rank', i): r['local_us'] for i, r in enumerate(recs)}
        if not by_rank:
            continue
        n_iter = min(len(v) for v in by_rank.values())
        wins = Counter(max(by_rank, key=lambda rk: by_rank[rk][i]) for i in range(n_iter))
        med = statistics.median(recs[0]['rank_max_us'])
        out.append({**{k: key[idx[k]] for k in CASE_KEYS}, 'slowest_rank_counts': dict(sorted(wins.items())),
                    'effective_gbps': round(max(r['bytes'] for r in recs) / (med * 1e-6) / 1e9, 1)})
    return out


def main(argv=None):
    p = argparse.ArgumentParser()
    p.add_argument('results')
    p.add_argument('--json', default='')
    args = p.parse_args(argv)
    groups = load_timings(args.results)
    fits, hist = sweep_fits(groups), bottleneck_ranks(groups)
    for f in fits:
        print(f"{f['model']:10s} {f['dispatch_dtype']:4s} {f['routing']:10s} {f['op']:16s} tokens {f['tokens']}: "
              f"latency {f['latency_us']} us, bandwidth {f['bandwidth_gbps']} GB/s, R2 {f['r2']}")
    for h in hist:
        print(f"{h['model']} T={h['tokens_per_rank']} {h['op']}: slowest rank counts {h['slowest_rank_counts']}, "
              f"{h['effective_gbps']} GB/s at the bottleneck rank")
    if args.json:
        with open(args.json, 'w') as fh:
            json.dump({'fits': fits, 'bottleneck_ranks': hist}, fh, indent=1)
    return 0


if __name__ == '__main__':
    raise SystemExit(main())
