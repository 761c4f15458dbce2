"""Markdown summary of `bench.py` JSON lines against the measured peaks and the published baseline.

    python bench.py > bench.json && python -m deepep_slingshot_b200.harness.report bench.json [more.json ...]

For every line: the headline (aggregate GB/s, per-rank GB/s, the ratio to the published SM100 EP8
figure), dispatch / combine per rank against the measured NVLink peer-copy bandwidth, the
low-latency latencies against the reference's published µs, the MoE step against its roofline,
the end-to-end number with its host transfers, and the SM clocks seen during the timed region.
Lines from several GPU counts are also put side by side (per-GPU value and its ratio to the
smallest run's per-GPU value, the weak-scaling efficiency).
"""
import argparse
import json
import os
import sys
from typing import Dict, List, Optional

PUBLISHED = {'dispatch_gbps_per_rank': 726.0, 'combine_gbps_per_rank': 740.0, 'cycle_gbps_per_rank': 735.1,
             'll_dispatch_us': 77.0, 'll_combine_us': 114.0}
NVLINK_GBPS = 770.0  # measured peer copy per direction on this pool


def load_lines(paths: List[str]) -> List[dict]:
    """JSON objects of every line that parses and carries a metric (other output is skipped)."""
    out = []
    for p in paths:
        with open(p) as f:
            for line in f:
                line = line.strip()
                if not line.startswith('{'):
                    continue
                try:
                    rec = json.loads(line)
                except json.JSONDecodeError:
                    continue
                if 'metric' in rec or 'unavailable' in rec:
                    out.append(rec)
    return out


def _fmt(v, nd=1) -> str:
    return '—' if v is None else (f'{v:.{nd}f}' if isinstance(v, float) else str(v))


def summarize(rec: dict, peaks: Optional[dict] = None) -> List[str]:
    """Markdown rows (| what | value | reference point |) of one bench line."""
    if 'unavailable' in rec:
        return [f"| {rec.get('impl', '?')} arm | unavailable | {rec['unavailable']} |"]
    n = rec.get('n_gpus', 1)
    rows = [f"| aggregate dispatch+combine | {_fmt(rec.get('value'))} GB/s over {n} GPU(s) | "
            f"{_fmt(rec.get('vs_baseline'), 3)} of {PUBLISHED['cycle_gbps_per_rank']} GB/s x {n} (published SM100 EP8) |"]
    for k in ('dispatch', 'combine'):
        v = rec.get(f'{k}_gbps_per_rank')
        if v is not None:
            rows.append(f"| {k} per rank | {_fmt(v)} GB/s ({_fmt(rec.get(f'{k}_ms', 0) * 1e3)} µs) | "
                        f"{v / PUBLISHED[f'{k}_gbps_per_rank']:.2f} of published {PUBLISHED[f'{k}_gbps_per_rank']:.0f}; "
                        f"{v / NVLINK_GBPS:.2f} of the {NVLINK_GBPS:.0f} GB/s peer copy |")
    if rec.get('dispatch_nosync_ms') is not None:
        alone = rec.get('dispatch_synced_alone_ms')
        rows.append(f"| dispatch host sync | step interval {_fmt(rec.get('dispatch_ms', 0) * 1e3)} µs"
                    + (f", synced alone {_fmt(alone * 1e3)} µs" if alone is not None else '')
                    + f", without the CPU sync {_fmt(rec['dispatch_nosync_ms'] * 1e3)} µs | "
                    "the synced dispatch's host round trip and the coupling of the ranks' host loops |")
    for k in ('ll_dispatch_us', 'll_combine_us'):
        v = rec.get(k)
        if v is not None:
            rows.append(f"| {k.replace('_us', '').replace('_', ' ')} | {_fmt(v)} µs | {PUBLISHED[k] / v:.2f}x faster than "
                        f"the published {PUBLISHED[k]:.0f} µs |")
    if rec.get('ll_moe_forward_us') is not None:
        rows.append(f"| decode MoE layer forward | {_fmt(rec['ll_moe_forward_us'])} µs | fused paths |")
    if rec.get('moe_tokens_per_s') is not None:
        roof = rec.get('moe_roofline_ms') or {}
        rows.append(f"| MoE fwd+bwd | {_fmt(rec['moe_tokens_per_s'], 0)} tok/s ({_fmt(rec.get('moe_ms_per_step'))} ms) | "
                    f"{_fmt(rec.get('moe_roofline_fraction'), 3)} of the roofline (bound {_fmt(roof.get('bound'))} ms: "
                    f"compute {_fmt(roof.get('compute'))}, NVLink {_fmt(roof.get('nvlink'))}, HBM {_fmt(roof.get('hbm'))}) |")
        hot = rec.get('moe_roofline_rank')
        if hot:
            rows.append(f"| MoE bounding rank | rank {hot.get('rank')}: {_fmt(hot.get('expert_rows'), 0)} expert rows | "
                        f"mean {_fmt(hot.get('expert_rows_mean'), 0)} rows per rank; remote tokens in "
                        f"{_fmt(hot.get('remote_tokens_in'), 0)}, out {_fmt(hot.get('remote_tokens_out'), 0)} |")
    e2e = rec.get('e2e')
    if e2e:
        rows.append(f"| end to end | {_fmt(e2e.get('value'))} GB/s ({_fmt(e2e.get('ms_per_step'), 3)} ms/step) | "
                    f"{e2e.get('schedule', '').split(':')[0]}; H2D {e2e.get('h2d_bytes_per_step', 0) / 1e6:.1f} MB/step"
                    + (f"; serial {_fmt(e2e['serial_value'])} GB/s" if e2e.get('serial_value') else '') + ' |')
    clocks = rec.get('clocks')
    if clocks:
        rows.append(f"| SM clock under load | {_fmt(clocks.get('sm_mhz'), 0)} / {_fmt(clocks.get('sm_max_mhz'), 0)} MHz | "
                    f"reasons: {', '.join(clocks.get('reasons') or []) or 'none'} |")
    if peaks:
        rows.append(f"| measured peaks | HBM {peaks.get('hbm_gbs')} GB/s, bf16 {peaks.get('bf16_tflops')} TFLOP/s | "
                    f"{peaks.get('gpu_name', '')} |")
    return rows


def scaling(recs: List[dict]) -> List[str]:
    """Per-GPU values across GPU counts and the weak-scaling efficiency to the smallest run."""
    runs = sorted((r for r in recs if 'value' in r and r.get('impl', 'ours') == 'ours'), key=lambda r: r.get('n_gpus', 1))
    if len(runs) < 2:
        return []
    base = runs[0]['value'] / runs[0].get('n_gpus', 1)
    out = ['', '| GPUs | aggregate GB/s | per GPU | efficiency vs smallest |', '|---|---|---|---|']
    for r in runs:
        n = r.get('n_gpus', 1)
        out.append(f"| {n} | {r['value']:.1f} | {r['value'] / n:.1f} | {r['value'] / n / base:.2f} |")
    return out


def main(argv=None) -> int:
    p = argparse.ArgumentParser()
    p.add_argument('files', nargs='+')
    p.add_argument('--peaks', default=None, help='MEASURED_PEAKS.json (default: next to bench.py)')
    args = p.parse_args(argv)
    recs = load_lines(args.files)
    if not recs:
        print('no bench lines found')
        return 1
    peaks_path = args.peaks or os.path.join(os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))),
                                            'MEASURED_PEAKS.json')
    peaks: Optional[Dict] = None
    if os.path.exists(peaks_path):
        with open(peaks_path) as f:
            peaks = json.load(f)
    for rec in recs:
        print(f"### {rec.get('impl', 'ours')}, {rec.get('n_gpus', '?')} GPU(s)\n")
        print('| what | value | reference point |\n|---|---|---|')
        for row in summarize(rec, peaks):
            print(row)
        print()
    for row in scaling(recs):
        print(row)
    return 0


if __name__ == '__main__':
    sys.exit(main())
