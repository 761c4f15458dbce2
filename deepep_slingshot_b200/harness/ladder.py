"""Qualification ladder: serial gates over the EP benchmark, each validated fail-closed before the
next one runs (the reference's gate controller, harness/runner/controller.py:36-125, and its ladders:
irregular stress, 4K correctness FP8 + BF16, dropped tokens, sustained 16K, performance with
counterbalanced repeats). A gate with `compare_with` must also reproduce an earlier gate's medians
within `max_rel_diff` (the repeat runs the models in the opposite order, so drift over time shows).

    torchrun --nproc-per-node 8 --master-addr 127.0.0.1 -m deepep_slingshot_b200.harness.ladder --out ladder_ep8

State lives in `<out>/ladder_state.json`: a gate that passed is skipped on the next run; after a
failure the ladder stops, and it runs again only with `--resume "<reason>"` (the reason is recorded)
and only if a read-only GPU health check (`utils/gpu_health.py`: uncorrected ECC errors, pending
page retirement or row remapping, hardware or thermal slowdown) finds nothing wrong.
"""
import argparse
import json
import os
import sys
import time
from typing import Callable, Dict, List, Optional

GATES: List[Dict] = [
    {'name': 'stress_small', 'args': ['--models', 'v4flash', 'qwen3', '--tokens', '32', '257', '--dtype', 'fp8',
                                      '--routing', 'uniform', 'mixed', 'hot_rank', '--seeds', '0', '1', '2',
                                      '--iters', '3', '--warmup', '1'], 'max_cv': 10.0},
    {'name': 'correctness_4k', 'args': ['--models', 'v4flash', 'qwen3', 'minimax', '--tokens', '4096', '--dtype', 'fp8',
                                        'bf16', '--routing', 'uniform', 'mixed', 'skew2', '--iters', '3', '--warmup', '1'],
     'max_cv': 10.0},
    {'name': 'dropped_tokens', 'args': ['--models', 'v4flash', 'deepseek_v3', '--tokens', '4096', '--dtype', 'fp8',
                                        'bf16', '--routing', 'uniform', 'mixed', '--drop-every', '7', '--iters', '3',
                                        '--warmup', '1'], 'max_cv': 10.0},
    {'name': 'sustained_16k', 'args': ['--models', 'v4flash', '--tokens', '16384', '--dtype', 'fp8', '--routing',
                                       'uniform', 'mixed', '--seeds', '0', '1', '--iters', '20', '--warmup', '5'],
     'max_cv': 0.15},
    {'name': 'perf_4k', 'args': ['--models', 'deepseek_v3', 'v4flash', '--tokens', '4096', '--dtype', 'fp8',
                                 '--routing', 'uniform', 'mixed', '--seeds', '0', '1', '2', '--iters', '20',
                                 '--warmup', '5'], 'max_cv': 0.15},
    {'name': 'perf_4k_repeat', 'args': ['--models', 'v4flash', 'deepseek_v3', '--tokens', '4096', '--dtype', 'fp8',
                                        '--routing', 'mixed', 'uniform', '--seeds', '0', '1', '2', '--iters', '20',
                                        '--warmup', '5'], 'max_cv': 0.15, 'compare_with': 'perf_4k', 'max_rel_diff': 0.1},
]


def compare_summaries(dir_a: str, dir_b: str, max_rel_diff: float) -> List[str]:
    """Problems where a case's median differs between two gates' summary.csv by more than
    `max_rel_diff`, or where the gates cover different cases."""
    import csv
    keys = ('model', 'tokens_per_rank', 'ranks', 'dispatch_dtype', 'routing', 'seed', 'op')

    def load(d):
        path = os.path.join(d, 'summary.csv')
        if not os.path.exists(path):
            return None
        with open(path) as f:
            return {tuple(r[k] for k in keys): float(r['median_rank_max_us']) for r in csv.DictReader(f)}
    a, b = load(dir_a), load(dir_b)
    if a is None or b is None:
        return [f'missing summary.csv in {dir_a if a is None else dir_b}']
    if set(a) != set(b):
        return [f'the gates cover different cases ({len(set(a) ^ set(b))} differ)']
    problems = []
    for k in sorted(a):
        lo, hi = min(a[k], b[k]), max(a[k], b[k])
        if lo <= 0 or (hi - lo) / lo > max_rel_diff:
            problems.append(f'{k}: median {a[k]:.1f} vs {b[k]:.1f} us (more than {max_rel_diff:.0%} apart)')
    return problems


def load_state(path: str) -> dict:
    """The ladder state file (passed gates, the failed gate, resume reasons), or a fresh one."""
    if os.path.exists(path):
        with open(path) as f:
            return json.load(f)
    return {'passed': [], 'failed': None, 'resumes': []}


def save_state(path: str, state: dict) -> None:
    """Write the ladder state atomically (temporary file + rename)."""
    tmp = path + '.tmp'
    with open(tmp, 'w') as f:
        json.dump(state, f, indent=1)
    os.replace(tmp, path)


def run_ladder(out: str, run_gate: Callable[[dict, str], List[str]], gates: List[Dict] = GATES,
               resume_reason: Optional[str] = None, is_leader: bool = True,
               health_check: Optional[Callable[[], List[str]]] = None) -> bool:
    """Run the gates in order. `run_gate(gate, gate_dir)` runs one gate and returns its validation
    problems (empty = pass). A resume after a failed gate needs a reason and, when `health_check` is
    given, a clean GPU health report (its problem lines, empty = healthy); both are recorded.
    Returns True when every gate passed."""
    os.makedirs(out, exist_ok=True)
    state_path = os.path.join(out, 'ladder_state.json')
    state = load_state(state_path)
    if state['failed'] is not None:
        if not resume_reason:
            if is_leader:
                print(f"[ladder] gate {state['failed']} failed earlier; rerun with --resume \"<reason>\"", flush=True)
            return False
        health = health_check() if health_check is not None else []
        if health:
            if is_leader:
                print('[ladder] not resuming, GPU health check failed:\n  ' + '\n  '.join(health), flush=True)
            return False
        state['resumes'].append({'gate': state['failed'], 'reason': resume_reason, 'time': time.time(),
                                 'health_checked': health_check is not None})
        state['failed'] = None
    for gate in gates:
        if gate['name'] in state['passed']:
            continue
        problems = run_gate(gate, os.path.join(out, gate['name']))
        if not problems and gate.get('compare_with'):
            problems = compare_summaries(os.path.join(out, gate['compare_with']), os.path.join(out, gate['name']),
                                         gate.get('max_rel_diff', 0.1))
        if problems:
            state['failed'] = gate['name']
            state['problems'] = problems[:50]
            if is_leader:
                save_state(state_path, state)
                print(f"[ladder] gate {gate['name']} FAILED ({len(problems)} problems)", flush=True)
            return False
        state['passed'].append(gate['name'])
        if is_leader:
            save_state(state_path, state)
            print(f"[ladder] gate {gate['name']} passed", flush=True)
    return True


def _run_gate_distributed(gate: dict, gate_dir: str) -> List[str]:
    import torch
    import torch.distributed as dist
    from .ep_benchmark import main as bench_main
    from .validate import validate
    rc = bench_main(gate['args'] + ['--out', gate_dir])
    dist.barrier()
    problems = validate(gate_dir, max_cv=gate.get('max_cv', 0.1)) if dist.get_rank() == 0 else []
    if rc != 0 and not problems:
        problems = [f'benchmark exited with {rc}']
    flag = torch.tensor([len(problems)], device='cuda')
    dist.broadcast(flag, 0)
    return problems if dist.get_rank() == 0 else (['failed on rank 0'] if int(flag.item()) else [])


def main(argv=None):
    import datetime

    import torch
    import torch.distributed as dist
    p = argparse.ArgumentParser()
    p.add_argument('--out', default='ladder_out')
    p.add_argument('--resume', default=None, help='reason for resuming after a failed gate (recorded)')
    args = p.parse_args(argv)
    local = int(os.environ.get('LOCAL_RANK', '0'))
    torch.cuda.set_device(local)
    os.environ.setdefault('MASTER_ADDR', '127.0.0.1')
    dist.init_process_group('nccl', timeout=datetime.timedelta(seconds=300), device_id=torch.device('cuda', local))
    from ..utils import gpu_health
    ok = run_ladder(args.out, _run_gate_distributed, resume_reason=args.resume, is_leader=dist.get_rank() == 0,
                    health_check=lambda: gpu_health.unhealthy(gpu_health.snapshot()))
    dist.destroy_process_group()
    return 0 if ok else 1


if __name__ == '__main__':
    sys.exit(main())
