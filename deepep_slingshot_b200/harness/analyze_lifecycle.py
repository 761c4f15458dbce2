"""Audit buffer lifecycle logs (`DEEPEP_B200_LIFECYCLE_LOG`) for leaks over create/destroy cycles.

    python -m deepep_slingshot_b200.harness.analyze_lifecycle 'lifecycle-rank{rank}.jsonl' \
        --ranks 8 --cycles 20 [--kind Buffer] [--tolerance-mib 4]

A cycle is a stretch of the log in which the number of live objects of one kind goes from zero
back to zero. For each rank the audit fails (ValueError) when:
  * the rank logged no event of that kind;
  * an object is destroyed that was not created, or objects are still alive at the end;
  * the number of cycles differs from the expected one;
  * a construction took less device memory than it requested (the record does not measure what
    the object holds);
  * the device memory in use after a cycle grows beyond the first cycle's by more than the
    tolerance (the first cycle may load modules and allocate library workspaces once).
The reference's audit (backend/tools/analyze_lifecycle.py, its test
backend/tests/test_lifecycle_analysis.py:8-58) applies the same idea to NIC context pools.
"""
import argparse
import json
import sys
from typing import Dict, Iterable, List


def read_log(path: str) -> List[dict]:
    """Records of one lifecycle JSONL file."""
    with open(path) as f:
        return [json.loads(line) for line in f if line.strip()]


def audit_rank(records: Iterable[dict], rank: int, cycles: int, kind: str = 'Buffer',
               tolerance_bytes: int = 4 << 20) -> Dict[str, int]:
    """Audit one rank's records of one kind (see the module docstring); returns the cycle
    count, peak live objects, baseline and largest growth, or raises ValueError."""
    recs = [r for r in records if r.get('rank') == rank and r.get('kind') == kind]
    if not recs:
        raise ValueError(f'no {kind} lifecycle events for rank {rank}')
    live = set()
    after_cycle: List[int] = []
    peak = 0
    for i, r in enumerate(recs):
        if r['phase'] == 'create':
            if r['id'] in live:
                raise ValueError(f'rank {rank}: record {i} creates object {r["id"]}, which is already alive')
            live.add(r['id'])
            peak = max(peak, len(live))
            before = r.get('used_before_bytes')
            if before is not None and r['device_used_bytes'] - before + tolerance_bytes < r['requested_bytes']:
                raise ValueError(f'rank {rank}: record {i} took {r["device_used_bytes"] - before} bytes of device '
                                 f'memory but requested {r["requested_bytes"]}')
        elif r['phase'] == 'destroy':
            if r['id'] not in live:
                raise ValueError(f'rank {rank}: record {i} destroys object {r["id"]}, which was not created')
            live.remove(r['id'])
            if not live:
                after_cycle.append(int(r['device_used_bytes']))
        else:
            raise ValueError(f'rank {rank}: record {i} has unknown phase {r["phase"]!r}')
    if live:
        raise ValueError(f'rank {rank}: {len(live)} {kind} object(s) still alive at the end of the log')
    if len(after_cycle) != cycles:
        raise ValueError(f'rank {rank}: {len(after_cycle)} {kind} cycles logged, expected {cycles}')
    baseline = after_cycle[0]
    growth = max(u - baseline for u in after_cycle)
    if growth > tolerance_bytes:
        worst = max(range(len(after_cycle)), key=lambda c: after_cycle[c])
        raise ValueError(f'rank {rank}: device memory in use grows across {kind} cycles: +{growth} bytes '
                         f'after cycle {worst} (tolerance {tolerance_bytes})')
    return {'rank': rank, 'cycles': len(after_cycle), 'peak_alive': peak, 'baseline_bytes': baseline,
            'max_growth_bytes': growth}


def main(argv=None) -> int:
    p = argparse.ArgumentParser()
    p.add_argument('log', help="log path; '{rank}' is replaced by each rank")
    p.add_argument('--ranks', type=int, default=1)
    p.add_argument('--cycles', type=int, required=True)
    p.add_argument('--kind', default='Buffer')
    p.add_argument('--tolerance-mib', type=float, default=4.0)
    args = p.parse_args(argv)
    ok = True
    for rank in range(args.ranks):
        try:
            records = read_log(args.log.replace('{rank}', str(rank)))
            print(json.dumps(audit_rank(records, rank, args.cycles, args.kind, int(args.tolerance_mib * (1 << 20)))))
        except (OSError, ValueError, KeyError) as e:
            ok = False
            print(f'FAIL rank {rank}: {e}')
    print('VALID' if ok else 'INVALID')
    return 0 if ok else 1


if __name__ == '__main__':
    sys.exit(main())
