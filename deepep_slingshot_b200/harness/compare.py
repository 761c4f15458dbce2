"""Paired A/B comparison of two `ep_benchmark` result directories.

    python -m deepep_slingshot_b200.harness.compare results_a results_b [--allow-other-host]

An A/B number is only meaningful when both runs moved the same bytes on the same placement. The
reference pairs its stock-dispatcher and adapter runs the same way before comparing them
(backend/tools/compare_sglang.py, tested by backend/tests/test_sglang_pairing.py): identical
inputs, routes and weights per rank and case, the same host and job placement, an exact reference
check passed in both. Here, per rank, the pairing fails (ValueError) when:
  * either run lacks the rank's manifest or correctness records;
  * the world sizes, hosts (unless allowed), GPU models or library versions differ;
  * the runs checked different cases, or a case's input / route hash differs between the runs;
  * a case did not pass its correctness check in both runs.
Differences that ARE the experiment (source hashes, `DEEPEP_*` / `NCCL_*` environment) are listed
in the result, not rejected. Then, per case and operation, the median rank-max times of both runs
(from their `summary.csv`) give `speedup = median_a / median_b`.
"""
import argparse
import csv
import glob
import json
import os
import sys
from typing import Dict, List, Tuple

CASE_ID = ('model', 'tokens_per_rank', 'ranks', 'dispatch_dtype', 'routing', 'seed')
PLACEMENT = ('world', 'gpu', 'torch', 'cuda', 'nccl', 'python')


def _read_jsonl(path: str) -> List[dict]:
    with open(path) as f:
        return [json.loads(line) for line in f if line.strip()]


def _load_run(out_dir: str) -> Tuple[Dict[int, dict], Dict[int, Dict[tuple, dict]]]:
    manifests, cases = {}, {}
    for p in sorted(glob.glob(os.path.join(out_dir, 'manifest-rank*.jsonl'))):
        recs = _read_jsonl(p)
        if recs:
            manifests[int(recs[-1]['rank'])] = recs[-1]
    if not manifests:
        raise ValueError(f'{out_dir}: no manifest records')
    for r in manifests:
        p = os.path.join(out_dir, f'correctness-rank{r}.jsonl')
        if not os.path.exists(p):
            raise ValueError(f'{out_dir}: missing correctness-rank{r}.jsonl')
        cases[r] = {tuple(x[k] for k in CASE_ID): x for x in _read_jsonl(p) if x.get('kind') == 'correctness'}
    return manifests, cases


def match_rank(rank: int, man_a: dict, man_b: dict, cases_a: Dict[tuple, dict], cases_b: Dict[tuple, dict],
               allow_other_host: bool = False) -> dict:
    """Check that one rank's records of two runs are comparable; returns what differs on purpose."""
    for k in PLACEMENT + (() if allow_other_host else ('host',)):
        if man_a.get(k) != man_b.get(k):
            raise ValueError(f'rank {rank}: {k} differs ({man_a.get(k)!r} vs {man_b.get(k)!r})')
    if set(cases_a) != set(cases_b):
        raise ValueError(f'rank {rank}: the runs checked different cases '
                         f'(only in A: {sorted(set(cases_a) - set(cases_b))}, only in B: {sorted(set(cases_b) - set(cases_a))})')
    for key, a in cases_a.items():
        b = cases_b[key]
        for field in ('input_sha256', 'route_sha256'):
            if a.get(field) is None or a.get(field) != b.get(field):
                raise ValueError(f'rank {rank} case {key}: {field} differs or is missing')
        if a.get('passed') is not True or b.get('passed') is not True:
            raise ValueError(f'rank {rank} case {key}: no passed exact-reference check in both runs')
    src_a, src_b = man_a.get('sources', {}), man_b.get('sources', {})
    env_a, env_b = man_a.get('env', {}), man_b.get('env', {})
    return {'changed_sources': sorted(k for k in set(src_a) | set(src_b) if src_a.get(k) != src_b.get(k)),
            'changed_env': sorted(k for k in set(env_a) | set(env_b) if env_a.get(k) != env_b.get(k))}


def _summary(out_dir: str) -> Dict[tuple, dict]:
    path = os.path.join(out_dir, 'summary.csv')
    if not os.path.exists(path):
        raise ValueError(f'{out_dir}: missing summary.csv')
    with open(path) as f:
        rows = list(csv.DictReader(f))
    return {tuple(r[k] for k in CASE_ID + ('op',)): r for r in rows}


def compare(dir_a: str, dir_b: str, allow_other_host: bool = False) -> Tuple[dict, List[dict]]:
    """Pair two result directories rank by rank (see the module docstring); returns the differences
    that are the experiment (changed sources / env) and the per-case paired rows."""
    man_a, cases_a = _load_run(dir_a)
    man_b, cases_b = _load_run(dir_b)
    if sorted(man_a) != sorted(man_b):
        raise ValueError(f'the runs have different ranks: {sorted(man_a)} vs {sorted(man_b)}')
    diffs = {}
    for r in sorted(man_a):
        d = match_rank(r, man_a[r], man_b[r], cases_a[r], cases_b[r], allow_other_host)
        for k, v in d.items():
            diffs.setdefault(k, set()).update(v)
    sum_a, sum_b = _summary(dir_a), _summary(dir_b)
    if set(sum_a) != set(sum_b):
        raise ValueError('the summaries cover different cases or operations')
    rows = []
    for key in sorted(sum_a):
        a, b = sum_a[key], sum_b[key]
        ma, mb = float(a['median_rank_max_us']), float(b['median_rank_max_us'])
        row = dict(zip(CASE_ID + ('op',), key))
        row.update({'median_us_a': ma, 'median_us_b': mb, 'speedup_b_over_a': round(ma / mb, 4) if mb > 0 else None,
                    'gbps_per_rank_a': float(a['gbps_per_rank']), 'gbps_per_rank_b': float(b['gbps_per_rank'])})
        rows.append(row)
    return {k: sorted(v) for k, v in diffs.items()}, rows


def main(argv=None) -> int:
    p = argparse.ArgumentParser()
    p.add_argument('dir_a')
    p.add_argument('dir_b')
    p.add_argument('--allow-other-host', action='store_true')
    p.add_argument('--out', default=None, help='CSV of the paired rows')
    args = p.parse_args(argv)
    try:
        diffs, rows = compare(args.dir_a, args.dir_b, args.allow_other_host)
    except (OSError, ValueError, KeyError) as e:
        print(f'NOT COMPARABLE: {e}')
        return 1
    print(f"changed sources: {len(diffs['changed_sources'])}, changed env: {diffs['changed_env']}")
    for r in rows:
        print(f"{r['model']:12s} {r['tokens_per_rank']:>6s} {r['dispatch_dtype']:4s} {r['routing']:8s} s{r['seed']} "
              f"{r['op']:16s} {r['median_us_a']:9.1f} -> {r['median_us_b']:9.1f} us  x{r['speedup_b_over_a']}")
    if args.out:
        with open(args.out, 'w', newline='') as f:
            wr = csv.DictWriter(f, fieldnames=list(rows[0].keys()))
            wr.writeheader()
            wr.writerows(rows)
    return 0


if __name__ == '__main__':
    sys.exit(main())
