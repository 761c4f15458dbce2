"""Size-sweep fit and bottleneck-rank histogram (`harness/analyze_sweep.py`) on synthetic benchmark
records with a known latency and bandwidth (CPU)."""
import json
import os

import pytest

from deepep_slingshot_b200.harness import analyze_sweep


def _write(dirpath, rank, recs):
    with open(os.path.join(dirpath, f'timings-rank{rank}.jsonl'), 'w') as f:
        for r in recs:
            f.write(json.dumps(r) + '\n')


def test_fit_recovers_latency_and_bandwidth(tmp_path):
    lat_us, gbps = 30.0, 400.0
    for rank in range(2):
        recs = []
        for tok in (128, 512, 2048, 8192):
            nbytes = tok * 8192 * (1 + rank)  # rank 1 moves twice the bytes (the bottleneck)
            t = lat_us + (tok * 8192 * 2) / (gbps * 1e3)   # µs for the bottleneck rank's bytes
            local = [t * (0.9 if rank == 0 else 1.0)] * 5
            local[2] = t * 1.2 if rank == 0 else t       # one iteration where rank 0 is slower
            recs.append({'kind': 'timing', 'rank': rank, 'model': 'mixtral', 'tokens_per_rank': tok, 'ranks': 2,
                         'dispatch_dtype': 'bf16', 'routing': 'uniform', 'seed': 0, 'op': 'dispatch',
                         'bytes': nbytes, 'local_us': local, 'rank_max_us': [t] * 5})
        _write(str(tmp_path), rank, recs)
    groups = analyze_sweep.load_timings(str(tmp_path))
    (fit,) = analyze_sweep.sweep_fits(groups)
    assert fit['tokens'] == [128, 512, 2048, 8192]
    assert fit['latency_us'] == pytest.approx(lat_us, rel=1e-3)
    assert fit['bandwidth_gbps'] == pytest.approx(gbps, rel=1e-3) and fit['r2'] == pytest.approx(1.0)
    hist = analyze_sweep.bottleneck_ranks(groups)
    assert len(hist) == 4 and all(h['slowest_rank_counts'] == {0: 1, 1: 4} for h in hist)


def test_fit_line_needs_two_sizes():
    with pytest.raises(ValueError):
        analyze_sweep.fit_line([1.0, 1.0], [2.0, 3.0])
