"""Fail-closed validators of a bench.py line and an nvlink_probe report (`harness/validate.py`)."""
import copy
import json

from deepep_slingshot_b200.harness.validate import main, validate_bench_line, validate_probe

LINE = {"metric": "m", "value": 497.0, "unit": "GB/s", "n_gpus": 1, "steps": 20, "warmup": 5, "ms_per_step": 0.19,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": 0.68, "dtype": "bf16", "data": "synthetic",
        "impl": "ours",
        "config": {"model": "x", "global_batch": 4096, "seq_len": 4096, "parallelism": "ep1", "l2": "flushed"},
        "clocks": {"sm_mhz": 1965.0, "sm_max_mhz": 1965.0, "reasons": ["sw_power_cap"]},
        "e2e": {"value": 80.7, "unit": "GB/s", "h2d_bytes_per_step": 59113472, "d2h_bytes_per_step": 4},
        "gpu_launches": 80}


def test_bench_line_contract():
    assert validate_bench_line(LINE) == []   # sw_power_cap is noted, not a failure
    bad = copy.deepcopy(LINE)
    del bad['gpu_launches']
    assert validate_bench_line(bad) == ['missing key gpu_launches']
    bad = copy.deepcopy(LINE)
    bad['clocks']['reasons'] = ['hw_thermal_slowdown']
    assert any('slowdown' in p for p in validate_bench_line(bad))
    bad = copy.deepcopy(LINE)
    bad['warmup'], bad['gpu_launches'] = 1, 0
    assert len(validate_bench_line(bad)) == 2
    bad = copy.deepcopy(LINE)
    bad['e2e']['h2d_bytes_per_step'] = 0
    assert validate_bench_line(bad) == ['e2e copies no inputs from the host']
    assert validate_bench_line({'impl': 'reference', 'unavailable': 'why'}) == []


def test_probe_report():
    rep = {'world': 2, 'flag_round_trip_ns': {'1': 4033.9},
           'store_sweep': [{'bytes': 4096, 'offset': 0, 'gbps': 0.5}], 'load_sweep': [{'bytes': 4096, 'offset': 0, 'gbps': 0.4}],
           'store_matrix_gbps': [[2800, 680], [690, 2760]], 'load_matrix_gbps': [[2790, 640], [650, 2810]]}
    assert validate_probe(rep) == []
    bad = dict(rep, load_matrix_gbps=[[1, 0], [1, 1]])
    assert validate_probe(bad) == ['load_matrix_gbps is not a complete 2 x 2 matrix of positive rates']
    assert validate_probe(dict(rep, flag_round_trip_ns={})) == ['round trips for 0 peers, expected 1']


def test_cli_kinds(tmp_path):
    b = tmp_path / 'bench.log'
    b.write_text('NCCL version x\n' + json.dumps(LINE) + '\n')
    assert main([str(b), '--kind', 'bench']) == 0
    (tmp_path / 'empty.log').write_text('no line\n')
    assert main([str(tmp_path / 'empty.log'), '--kind', 'bench']) == 1
