"""Profile interval analysis (CPU): synthetic Chrome-trace events, a fabricated capture directory,
and a real CPU-only torch.profiler trace."""
import json
import math

import pytest
import torch

from deepep_slingshot_b200.harness import analyze_profiles as ap


def _events(op='cycle', iterations=1, corr=False):
    """Per iteration (100 µs apart): a 12 µs marker, three kernels (one overlapping another, one
    launched inside the marker but running after it) and a 20 µs device synchronisation."""
    ev = []
    for i in range(iterations):
        t = 100.0 * i
        ev.append({'ph': 'X', 'cat': 'user_annotation', 'name': f'ep/{op}/iteration{i}', 'ts': t, 'dur': 12})
        kernels = [('stage', 3, 9), ('notify', 5, 4), ('pull', 16, 3)]
        for j, (name, s, d) in enumerate(kernels):
            c = 1000 * i + j
            ev.append({'ph': 'X', 'cat': 'kernel', 'name': name, 'ts': t + s, 'dur': d, 'args': {'correlation': c}})
            if corr:
                ev.append({'ph': 'X', 'cat': 'cuda_runtime', 'name': 'cudaLaunchKernel', 'ts': t + 1 + j, 'dur': 1,
                           'args': {'correlation': c}})
        ev.append({'ph': 'X', 'cat': 'cuda_runtime', 'name': 'cudaDeviceSynchronize', 'ts': t + 2, 'dur': 20})
    return ev


@pytest.mark.parametrize('corr', [False, True])
def test_span_union_gap_overlap(corr):
    rows, kernels = ap.analyze_events(_events(iterations=2, corr=corr), 'cycle', 2)
    assert len(rows) == 2
    for r in rows:
        assert r['kernels'] == 3
        assert r['kernel_span_us'] == 16       # 3 .. 19
        assert r['kernel_union_us'] == 12      # [3, 12] + [16, 19]
        assert r['kernel_gap_us'] == 4
        assert r['kernel_overlap_us'] == 4     # notify [5, 9] inside stage
        assert r['sync_api_union_us'] == 20
    assert [k['kernel'] for k in kernels] == ['stage', 'notify', 'pull']
    assert kernels[0]['calls'] == 2 and kernels[0]['total_us'] == 18


def test_correlation_beats_windows():
    """A kernel whose launch lies in iteration 0's range counts there even if it runs after
    iteration 1 began."""
    ev = _events(iterations=2, corr=True)
    late = {'ph': 'X', 'cat': 'kernel', 'name': 'late', 'ts': 150.0, 'dur': 5, 'args': {'correlation': 77}}
    ev += [late, {'ph': 'X', 'cat': 'cuda_runtime', 'name': 'cudaLaunchKernel', 'ts': 8, 'dur': 1,
                  'args': {'correlation': 77}}]
    rows, _ = ap.analyze_events(ev, 'cycle', 2)
    assert rows[0]['kernels'] == 4 and rows[1]['kernels'] == 3


def test_rejections():
    with pytest.raises(ValueError, match='No GPU'):
        ap.analyze_events([_events()[0]], 'cycle', 1)
    with pytest.raises(ValueError, match='iteration 1'):
        ap.analyze_events(_events(), 'cycle', 2)
    with pytest.raises(ValueError, match='iteration 0'):
        ap.analyze_events(_events(op='combine'), 'cycle', 1)
    for bad in ([(2.0, 1.0)], [(0.0, math.nan)], [(0.0, math.inf)]):
        with pytest.raises(ValueError, match='invalid interval'):
            ap.interval_stats(bad)
    assert ap.interval_stats([]) == {'span': 0.0, 'union': 0.0, 'gap': 0.0, 'overlap': 0.0, 'busy': 0.0}


def _capture_dir(tmp_path, world=2, ops=('dispatch', 'combine')):
    tmp_path.mkdir(parents=True, exist_ok=True)
    case = {'tokens': 4096, 'hidden': 7168, 'experts': 256, 'topk': 8, 'world': world, 'dtype': 'fp8'}
    for op in ops:
        for r in range(world):
            (tmp_path / f'{op}-rank{r}.json').write_text(json.dumps({'traceEvents': _events(op, 2, corr=True)}))
            c = dict(case, input_sha256=f'in{r}', route_sha256=f'route{r}')
            (tmp_path / f'{op}-rank{r}-summary.json').write_text(
                json.dumps({'operation': op, 'rank': r, 'profiled_iterations': 2, 'case': c}))
    return tmp_path


def test_capture_directory(tmp_path):
    status, rows, kernels = ap.analyze(str(_capture_dir(tmp_path)))
    assert status['status'] == 'DIAGNOSTIC_ONLY' and status['operations'] == ['combine', 'dispatch']
    assert len(rows) == 2 * 2 * 2 and len(kernels) == 2 * 2 * 3
    assert ap.main([str(tmp_path)]) == 0
    assert (tmp_path / 'profile_rows.csv').exists() and (tmp_path / 'profile_status.json').exists()


def test_capture_directory_rejections(tmp_path):
    d = _capture_dir(tmp_path / 'a')
    (d / 'combine-rank1-summary.json').unlink()
    with pytest.raises(ValueError, match='Missing traces for combine'):
        ap.analyze(str(d))
    d = _capture_dir(tmp_path / 'b')
    (d / 'dispatch-rank0.json').unlink()
    with pytest.raises(ValueError, match='Missing traces'):
        ap.analyze(str(d))
    d = _capture_dir(tmp_path / 'c')
    rec = json.loads((d / 'combine-rank1-summary.json').read_text())
    rec['case']['tokens'] = 8192
    (d / 'combine-rank1-summary.json').write_text(json.dumps(rec))
    with pytest.raises(ValueError, match='different correctness cases'):
        ap.analyze(str(d))
    assert ap.main([str(d)]) == 1
    with pytest.raises(ValueError, match='no profile summaries'):
        ap.analyze(str(tmp_path / 'empty_does_not_exist'))


def test_real_cpu_trace(tmp_path):
    """A torch.profiler trace of a CPU-only run has the markers but no device events; with one
    device event added inside the marker's window the iteration is analyzed."""
    with torch.profiler.profile(activities=[torch.profiler.ProfilerActivity.CPU]) as prof:
        for i in range(2):
            with torch.profiler.record_function(f'ep/cycle/iteration{i}'):
                torch.ones(64).sum()
    path = tmp_path / 't.json'
    prof.export_chrome_trace(str(path))
    events = json.loads(path.read_text())['traceEvents']
    with pytest.raises(ValueError, match='No GPU'):
        ap.analyze_events(events, 'cycle', 2)
    marks = sorted((e for e in events if e.get('ph') == 'X' and str(e.get('name', '')).startswith('ep/cycle/')),
                   key=lambda e: e['ts'])
    assert len(marks) == 2
    for m in marks:
        events.append({'ph': 'X', 'cat': 'kernel', 'name': 'k', 'ts': float(m['ts']), 'dur': 1.0})
    rows, _ = ap.analyze_events(events, 'cycle', 2)
    assert [r['kernels'] for r in rows] == [1, 1]
