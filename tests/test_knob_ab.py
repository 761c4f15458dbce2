"""CPU tests of the switch A/B harness (`harness/knob_ab.py`) with a fake child runner: parsing of the
workload timing lines, set-up workloads left out of the comparison, ratios to the first variant,
failed variants reported without stopping the set, and the table."""
from deepep_slingshot_b200.harness import knob_ab


def fake_runner(times_by_env):
    calls = []

    def run(env, workloads, reps, timeout):
        calls.append((dict(env), list(workloads), reps))
        key = tuple(sorted(env.items()))
        if key not in times_by_env:
            return 1, 'Traceback: boom\nRuntimeError: launch failed'
        lines = ['kernel workloads done: ' + ','.join(workloads)]
        for w, us in times_by_env[key].items():
            lines.append(f'time {w}: median {us:.1f} us, min {us * 0.9:.1f} us')
        return 0, '\n'.join(lines)
    return run, calls


def test_parse_times():
    t = knob_ab.parse_times('noise\ntime grouped_gemm: median 188.5 us, min 180.0 us\ntime x: median 1 us\n')
    assert t == {'grouped_gemm': {'median_us': 188.5, 'min_us': 180.0}}


def test_gemm_set_ratios_and_failures():
    run, calls = fake_runner({(): {'grouped_gemm': 200.0},
                              (('DEEPEP_B200_GEMM_BN', '128'),): {'grouped_gemm': 260.0},
                              (('DEEPEP_B200_GEMM_PAIR', '1'),): {'grouped_gemm': 280.0}})
    rows = knob_ab.run_set('gemm', reps=5, run=run)
    assert [c[0] for c in calls] == [v[1] for v in knob_ab.SETS['gemm']] and all(c[2] == 5 for c in calls)
    assert rows[0]['ratio_to_first'] == 1.0 and abs(rows[1]['ratio_to_first'] - 1.3) < 1e-9
    assert rows[3]['rc'] == 1 and rows[3]['total_median_us'] is None and 'launch failed' in rows[3]['tail']
    text = '\n'.join(knob_ab.table('gemm', rows))
    assert '| 128x128 tiles | DEEPEP_B200_GEMM_BN=128 | grouped_gemm | 260.0 | 1.300 |' in text
    assert 'failed (rc 1)' in text


def test_setup_workloads_are_not_compared():
    run, _ = fake_runner({(): {'dispatch': 90.0, 'combine': 80.0},
                          (('DEEPEP_B200_COMBINE_ANNOUNCE', 'lagged'),): {'dispatch': 95.0, 'combine': 60.0}})
    rows = knob_ab.run_set('combine', run=run)
    assert rows[0]['compared'] == ['combine'] and rows[0]['total_median_us'] == 80.0
    assert abs(rows[1]['ratio_to_first'] - 0.75) < 1e-9


def test_every_set_names_known_workloads():
    import ast
    import os
    src = open(os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
                            'deepep_slingshot_b200', 'utils', 'kernel_workloads.py')).read()
    names = set()
    for node in ast.walk(ast.parse(src)):
        if isinstance(node, ast.Dict):
            for k in node.keys:
                if isinstance(k, ast.Constant) and isinstance(k.value, str):
                    names.add(k.value)
    for variants in knob_ab.SETS.values():
        for _, env, workloads in variants:
            assert set(workloads) <= names, workloads
            assert all(k.startswith('DEEPEP_B200_') for k in env)
