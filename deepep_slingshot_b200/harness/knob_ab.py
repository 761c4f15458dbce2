"""A/B timing of the library's run-time switches on one GPU, one process per variant.

Every `DEEPEP_B200_*` switch is read once per process, so each variant runs
`python -m deepep_slingshot_b200.utils.kernel_workloads --only <workloads> --time <reps>` in a child
process with its environment, and the median CUDA-event times it prints (L2 flushed before every
repetition) are put side by side, as a ratio to the set's first variant:

    python -m deepep_slingshot_b200.harness.knob_ab --set gemm [--reps 20] [--json out.json]

Sets: `gemm` (FP8 grouped GEMM tile width and CTA-pair variants), `stage` (the dispatch stage's row
path, signalling scope and writer fence), `combine` (arrival announcements), `down_proj` (the down
projection followed by the weighted expanded combine against the down projection with the combine
send as its epilogue). A variant that fails reports its exit code and output tail and the others
still run.
"""
import argparse
import json
import os
import re
import subprocess
import sys
from typing import Callable, Dict, List, Optional

# set -> [(label, environment overrides, workloads)]; the first variant is the baseline
SETS: Dict[str, List[tuple]] = {
    'gemm': [('128x256 tiles (default)', {}, ['grouped_gemm']),
             ('128x128 tiles', {'DEEPEP_B200_GEMM_BN': '128'}, ['grouped_gemm']),
             ('CTA pairs, 16 epilogue warps', {'DEEPEP_B200_GEMM_PAIR': '1'}, ['grouped_gemm']),
             ('CTA pairs, 8 epilogue warps', {'DEEPEP_B200_GEMM_PAIR': '2'}, ['grouped_gemm'])],
    'stage': [('default', {}, ['dispatch']),
              ('rows through registers', {'DEEPEP_B200_STAGE_ROWS': 'regs'}, ['dispatch']),
              ('GPU-scope chunk counters', {'DEEPEP_B200_STAGE_SIGNAL_SCOPE': 'gpu'}, ['dispatch']),
              ('no writer proxy fence', {'DEEPEP_B200_STAGE_WRITER_FENCE': '0'}, ['dispatch']),
              ('stage warps in the pull', {'DEEPEP_B200_DISPATCH_STAGE': 'warps'}, ['dispatch'])],
    'combine': [('drain per batch (default)', {}, ['dispatch', 'combine']),
                ('lagged announcements', {'DEEPEP_B200_COMBINE_ANNOUNCE': 'lagged'}, ['dispatch', 'combine'])],
    'down_proj': [('grouped GEMM, then the weighted expanded combine', {}, ['gemm_then_combine']),
                  ('GEMM with the combine send as its epilogue + reduce', {}, ['gemm_combine'])],
}

_TIME = re.compile(r'^time (\w+): median ([0-9.]+) us, min ([0-9.]+) us')


def parse_times(text: str) -> Dict[str, Dict[str, float]]:
    """{workload: {'median_us', 'min_us'}} from kernel_workloads' `time` lines."""
    out = {}
    for line in text.splitlines():
        m = _TIME.match(line.strip())
        if m:
            out[m.group(1)] = {'median_us': float(m.group(2)), 'min_us': float(m.group(3))}
    return out


def _run_child(env_overrides: Dict[str, str], workloads: List[str], reps: int, timeout: float):
    env = dict(os.environ)
    env.update(env_overrides)
    cmd = [sys.executable, '-m', 'deepep_slingshot_b200.utils.kernel_workloads', '--only', ','.join(workloads),
           '--time', str(reps)]
    try:
        p = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=timeout)
        return p.returncode, p.stdout + p.stderr
    except subprocess.TimeoutExpired as e:
        return -1, f'timed out after {timeout} s: {e}'


def run_set(name: str, reps: int = 20, timeout: float = 600.0,
            run: Optional[Callable[[Dict[str, str], List[str], int, float], tuple]] = None) -> List[dict]:
    """One record per variant: label, environment, workloads, per-workload medians, the summed median
    of the variant's timed workloads (the ones its set compares) and the ratio to the first variant."""
    run = run or _run_child
    rows = []
    for label, env, workloads in SETS[name]:
        rc, text = run(env, workloads, reps, timeout)
        times = parse_times(text)
        # workloads a variant needs only as set-up (dispatch before combine) are not compared
        compared = [w for w in workloads if w in times and not (w == 'dispatch' and len(workloads) > 1)]
        total = sum(times[w]['median_us'] for w in compared) if rc == 0 and compared else None
        rows.append({'label': label, 'env': env, 'workloads': workloads, 'rc': rc, 'times': times,
                     'compared': compared, 'total_median_us': total,
                     'tail': '' if rc == 0 else text[-800:]})
    base = rows[0]['total_median_us'] if rows else None
    for r in rows:
        r['ratio_to_first'] = (r['total_median_us'] / base) if base and r['total_median_us'] else None
    return rows


def table(name: str, rows: List[dict]) -> List[str]:
    out = [f'### {name}', '', '| variant | environment | timed workloads | median µs | vs first |', '|---|---|---|---|---|']
    for r in rows:
        env = ' '.join(f'{k}={v}' for k, v in r['env'].items()) or '(none)'
        if r['total_median_us'] is None:
            out.append(f"| {r['label']} | {env} | {', '.join(r['workloads'])} | failed (rc {r['rc']}) | – |")
        else:
            out.append(f"| {r['label']} | {env} | {', '.join(r['compared'])} | {r['total_median_us']:.1f} | "
                       f"{r['ratio_to_first']:.3f} |")
    return out


def main(argv=None) -> int:
    p = argparse.ArgumentParser()
    p.add_argument('--set', action='append', choices=sorted(SETS), required=True)
    p.add_argument('--reps', type=int, default=20)
    p.add_argument('--timeout', type=float, default=600.0)
    p.add_argument('--json', default='')
    args = p.parse_args(argv)
    results = {}
    for name in args.set:
        rows = run_set(name, args.reps, args.timeout)
        results[name] = rows
        print('\n'.join(table(name, rows)))
        for r in rows:
            if r['tail']:
                print(f"[{r['label']}] rc {r['rc']}:\n{r['tail']}")
    if args.json:
        with open(args.json, 'w') as f:
            json.dump(results, f, indent=1)
    return 0 if all(r['rc'] == 0 for rows in results.values() for r in rows) else 1


if __name__ == '__main__':
    raise SystemExit(main())
