"""Paired A/B comparison of two benchmark result directories (CPU, fabricated records)."""
import copy
import csv
import json

import pytest

from deepep_slingshot_b200.harness import compare as cmp

CASES = [('v4flash', 4096, 2, 'fp8', 'uniform', 0), ('v4flash', 4096, 2, 'fp8', 'mixed', 0)]


def _write_run(d, world=2, host='node-a', env=None, sources=None, hashes='same', passed=True, medians=None):
    d.mkdir(parents=True)
    for r in range(world):
        man = {'kind': 'manifest', 'rank': r, 'world': world, 'host': host, 'gpu': 'NVIDIA B200', 'torch': '2.11',
               'cuda': '12.8', 'nccl': '2.28.9', 'python': '3.12.3', 'env': env or {'DEEPEP_B200_ROW_CHUNK': '0'},
               'sources': sources or {'csrc/kernels/intranode.cu': 'abc'}}
        (d / f'manifest-rank{r}.jsonl').write_text(json.dumps(man) + '\n')
        with open(d / f'correctness-rank{r}.jsonl', 'w') as f:
            for c in CASES:
                rec = dict(zip(cmp.CASE_ID, c), kind='correctness', passed=passed,
                           input_sha256=f'in-{r}-{c[4]}-{hashes}', route_sha256=f'route-{r}-{c[4]}')
                f.write(json.dumps(rec) + '\n')
    medians = medians or {}
    with open(d / 'summary.csv', 'w', newline='') as f:
        w = csv.DictWriter(f, fieldnames=list(cmp.CASE_ID) + ['op', 'median_rank_max_us', 'gbps_per_rank'])
        w.writeheader()
        for c in CASES:
            for op in ('dispatch', 'combine'):
                m = medians.get((c[4], op), 100.0)
                w.writerow(dict(zip(cmp.CASE_ID, c), op=op, median_rank_max_us=m, gbps_per_rank=round(1e4 / m, 1)))
    return d


def test_paired_speedups(tmp_path):
    a = _write_run(tmp_path / 'a')
    b = _write_run(tmp_path / 'b', env={'DEEPEP_B200_ROW_CHUNK': '4'}, sources={'csrc/kernels/intranode.cu': 'def'},
                   medians={('uniform', 'combine'): 80.0})
    diffs, rows = cmp.compare(str(a), str(b))
    assert diffs == {'changed_sources': ['csrc/kernels/intranode.cu'], 'changed_env': ['DEEPEP_B200_ROW_CHUNK']}
    assert len(rows) == 4
    comb = next(r for r in rows if r['routing'] == 'uniform' and r['op'] == 'combine')
    assert comb['speedup_b_over_a'] == 1.25
    assert all(r['speedup_b_over_a'] == 1.0 for r in rows if r is not comb)
    out = tmp_path / 'paired.csv'
    assert cmp.main([str(a), str(b), '--out', str(out)]) == 0 and out.exists()


@pytest.mark.parametrize('kw,match', [
    ({'hashes': 'other'}, 'input_sha256'),
    ({'host': 'node-b'}, 'host differs'),
    ({'passed': False}, 'passed exact-reference'),
    ({'world': 1}, 'different ranks'),
])
def test_not_comparable(tmp_path, kw, match):
    a = _write_run(tmp_path / 'a')
    b = _write_run(tmp_path / 'b', **kw)
    with pytest.raises(ValueError, match=match):
        cmp.compare(str(a), str(b))
    assert cmp.main([str(a), str(b)]) == 1


def test_other_host_allowed_and_field_checks(tmp_path):
    a = _write_run(tmp_path / 'a')
    b = _write_run(tmp_path / 'b', host='node-b')
    assert len(cmp.compare(str(a), str(b), allow_other_host=True)[1]) == 4
    man = json.loads((a / 'manifest-rank0.jsonl').read_text())
    cases = {tuple(c): {'input_sha256': 'x', 'route_sha256': 'y', 'passed': True} for c in CASES}
    other = copy.deepcopy(man)
    other['nccl'] = '2.27.3'
    with pytest.raises(ValueError, match='nccl differs'):
        cmp.match_rank(0, man, other, cases, cases)
    fewer = dict(list(cases.items())[:1])
    with pytest.raises(ValueError, match='different cases'):
        cmp.match_rank(0, man, man, cases, fewer)
    missing = {k: dict(v, route_sha256=None) for k, v in cases.items()}
    with pytest.raises(ValueError, match='route_sha256'):
        cmp.match_rank(0, man, man, missing, missing)


def test_missing_files(tmp_path):
    a = _write_run(tmp_path / 'a')
    b = _write_run(tmp_path / 'b')
    (b / 'correctness-rank1.jsonl').unlink()
    with pytest.raises(ValueError, match='missing correctness-rank1'):
        cmp.compare(str(a), str(b))
    c = _write_run(tmp_path / 'c')
    (c / 'summary.csv').unlink()
    with pytest.raises(ValueError, match='missing summary.csv'):
        cmp.compare(str(a), str(c))
    with pytest.raises(ValueError, match='no manifest'):
        cmp.compare(str(a), str(tmp_path / 'nothing'))
