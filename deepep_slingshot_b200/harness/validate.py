"""Fail-closed validation of an `ep_benchmark` results directory (and, with `--kind`, of a
`bench.py` line or an `nvlink_probe` report).

    python -m deepep_slingshot_b200.harness.validate ep_results [--max-cv 0.1] [--ranks 8]
    python -m deepep_slingshot_b200.harness.validate bench.log --kind bench
    python -m deepep_slingshot_b200.harness.validate probe.json --kind probe

Passes (exit 0) only when:
  * every rank wrote a manifest, and all manifests agree on the world size and the source hashes
    (the same code ran everywhere);
  * every correctness record passed, and every rank checked the same set of cases;
  * every checked case has timing records from every rank for each operation, with positive
    rank-max times;
  * `summary.csv` exists and, when seeds repeat, the median's coefficient of variation over seeds
    stays below `--max-cv`.
Any missing file or record fails the run (nothing is inferred). The reference's qualification
ladders validate their gates the same fail-closed way (backend/tools/validate_gate.py).
"""
import argparse
import glob
import json
import os
import sys
from collections import defaultdict
from typing import List


def _read_jsonl(path: str) -> List[dict]:
    with open(path) as f:
        return [json.loads(line) for line in f if line.strip()]


def validate(out_dir: str, max_cv: float = 0.1, ranks: int = 0) -> List[str]:
    """List of problems (empty = valid)."""
    problems = []
    manifests = sorted(glob.glob(os.path.join(out_dir, 'manifest-rank*.jsonl')))
    if not manifests:
        return [f'no manifest in {out_dir}']
    mans = {}
    for p in manifests:
        recs = _read_jsonl(p)
        if not recs:
            problems.append(f'{os.path.basename(p)} is empty')
            continue
        m = recs[-1]
        mans[m['rank']] = m
    worlds = {m['world'] for m in mans.values()}
    if len(worlds) != 1:
        problems.append(f'manifests disagree on the world size: {sorted(worlds)}')
    world = next(iter(worlds)) if worlds else 0
    if ranks and world != ranks:
        problems.append(f'world size {world}, expected {ranks}')
    if sorted(mans) != list(range(world)):
        problems.append(f'manifests from ranks {sorted(mans)}, expected 0..{world - 1}')
    hashes = {json.dumps(m.get('sources', {}), sort_keys=True) for m in mans.values()}
    if len(hashes) != 1:
        problems.append('ranks ran different source trees (source hashes differ)')

    cases_by_rank = {}
    for r in range(world):
        path = os.path.join(out_dir, f'correctness-rank{r}.jsonl')
        if not os.path.exists(path):
            problems.append(f'missing correctness-rank{r}.jsonl')
            continue
        recs = _read_jsonl(path)
        failed = [x for x in recs if not x.get('passed')]
        for x in failed:
            problems.append(f"rank {r}: correctness failed for {x.get('model')} {x.get('routing')} "
                            f"{x.get('dispatch_dtype')} seed {x.get('seed')}: {x.get('error', '')}")
        cases_by_rank[r] = {(x['model'], x['tokens_per_rank'], x['dispatch_dtype'], x['routing'], x['seed'])
                            for x in recs if x.get('passed')}
    if cases_by_rank and len({frozenset(v) for v in cases_by_rank.values()}) != 1:
        problems.append('ranks checked different sets of cases')

    timings = defaultdict(dict)
    for r in range(world):
        path = os.path.join(out_dir, f'timings-rank{r}.jsonl')
        if not os.path.exists(path):
            problems.append(f'missing timings-rank{r}.jsonl')
            continue
        for x in _read_jsonl(path):
            if x.get('kind') != 'timing':
                continue
            key = (x['model'], x['tokens_per_rank'], x['dispatch_dtype'], x['routing'], x['seed'])
            timings[key].setdefault(x['op'], {})[r] = x
    ops = ('dispatch', 'cached_dispatch', 'combine')
    for key in cases_by_rank.get(0, set()):
        for op in ops:
            per_rank = timings.get(key, {}).get(op, {})
            if sorted(per_rank) != list(range(world)):
                problems.append(f'{key} {op}: timings from ranks {sorted(per_rank)}')
                continue
            if any(min(x['rank_max_us']) <= 0 for x in per_rank.values()):
                problems.append(f'{key} {op}: non-positive times')

    summary = os.path.join(out_dir, 'summary.csv')
    if not os.path.exists(summary):
        problems.append('missing summary.csv')
    rep_path = os.path.join(out_dir, 'repeatability.json')
    if os.path.exists(rep_path):
        with open(rep_path) as f:
            for k, v in json.load(f).items():
                if len(v.get('medians_us', [])) > 1 and v.get('cv', 0.0) > max_cv:
                    problems.append(f'{k}: median varies over seeds (cv {v["cv"]} > {max_cv})')
    else:
        problems.append('missing repeatability.json')
    return problems


# The benchmark line's contract: the keys every `bench.py` JSON line carries for its driver.
BENCH_KEYS = ('metric', 'value', 'unit', 'n_gpus', 'steps', 'warmup', 'ms_per_step', 'higher_is_better', 'scaling',
              'vs_baseline', 'dtype', 'data', 'config', 'clocks', 'gpu_launches')
BENCH_CONFIG_KEYS = ('model', 'global_batch', 'seq_len', 'parallelism', 'l2')
THROTTLE_REASONS = ('hw_slowdown', 'hw_thermal_slowdown', 'sw_thermal_slowdown')


def validate_bench_line(line: dict) -> List[str]:
    """Fail-closed check of one `bench.py` line (this library's arm): contract keys, sane values,
    an end-to-end number with its host transfer bytes, kernels launched, and no thermal or hardware
    slowdown during the timed steps."""
    if line.get('impl') == 'reference' and 'unavailable' in line:
        return []  # the reference arm's documented unavailability line
    problems = [f'missing key {k}' for k in BENCH_KEYS if k not in line]
    cfg = line.get('config') or {}
    problems += [f'missing config.{k}' for k in BENCH_CONFIG_KEYS if k not in cfg]
    if problems:
        return problems
    if not (isinstance(line['value'], (int, float)) and line['value'] > 0):
        problems.append(f"value {line['value']!r} is not a positive number")
    if line['warmup'] < 3:
        problems.append(f"warmup {line['warmup']} < 3")
    if line['scaling'] not in ('weak', 'strong'):
        problems.append(f"scaling {line['scaling']!r}")
    if line.get('impl', 'ours') == 'ours':
        if not line['gpu_launches']:
            problems.append('gpu_launches is 0: no kernel of this library ran in the timed region')
        e2e = line.get('e2e')
        if e2e is not None:
            for k in ('value', 'unit', 'h2d_bytes_per_step', 'd2h_bytes_per_step'):
                if k not in e2e:
                    problems.append(f'missing e2e.{k}')
            if e2e.get('h2d_bytes_per_step', 0) <= 0:
                problems.append('e2e copies no inputs from the host')
    reasons = set((line['clocks'] or {}).get('reasons', []))
    bad = sorted(reasons & set(THROTTLE_REASONS))
    if bad:
        problems.append(f"clock slowdown during the timed steps: {', '.join(bad)}")
    return problems


def validate_probe(report: dict) -> List[str]:
    """Fail-closed check of an `nvlink_probe` report: a positive finite round trip per peer, a
    positive bandwidth in every sweep row, a complete per-pair matrix."""
    problems = []
    world = report.get('world')
    if not isinstance(world, int) or world < 1:
        return ['missing or bad world size']
    lat = report.get('flag_round_trip_ns') or {}
    if len(lat) != max(1, world - 1):
        problems.append(f'round trips for {len(lat)} peers, expected {max(1, world - 1)}')
    problems += [f'round trip to {k}: {v!r}' for k, v in lat.items() if not (isinstance(v, (int, float)) and 0 < v < 1e7)]
    for kind in ('store_sweep', 'load_sweep'):
        rows = report.get(kind)
        if not rows:
            problems.append(f'missing {kind}')
            continue
        problems += [f"{kind}: {r.get('bytes')} B at offset {r.get('offset')}: {r.get('gbps')!r} GB/s"
                     for r in rows if not (r.get('gbps') or 0) > 0]
    for kind in ('store_matrix_gbps', 'load_matrix_gbps'):
        m = report.get(kind)
        if not m or len(m) != world or any(len(row) != world or min(row) <= 0 for row in m):
            problems.append(f'{kind} is not a complete {world} x {world} matrix of positive rates')
    return problems


def main(argv=None):
    p = argparse.ArgumentParser()
    p.add_argument('out_dir', help='ep_benchmark results directory, bench.py output file (--kind bench) or '
                                   'nvlink_probe report (--kind probe)')
    p.add_argument('--kind', choices=['ep', 'bench', 'probe'], default='ep')
    p.add_argument('--max-cv', type=float, default=0.1)
    p.add_argument('--ranks', type=int, default=0)
    args = p.parse_args(argv)
    if args.kind == 'bench':
        with open(args.out_dir) as f:
            lines = [json.loads(l) for l in f if l.strip().startswith('{')]
        problems = ['no JSON line'] if not lines else [x for l in lines for x in validate_bench_line(l)]
    elif args.kind == 'probe':
        with open(args.out_dir) as f:
            problems = validate_probe(json.load(f))
    else:
        problems = validate(args.out_dir, args.max_cv, args.ranks)
    for x in problems:
        print('FAIL', x)
    print('VALID' if not problems else f'INVALID ({len(problems)} problems)')
    return 0 if not problems else 1


if __name__ == '__main__':
    sys.exit(main())
