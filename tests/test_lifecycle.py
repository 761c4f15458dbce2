"""Lifecycle records and their leak audit (CPU: synthetic logs; the device probe is faked)."""
import json

import pytest

from deepep_slingshot_b200.harness import analyze_lifecycle as al
from deepep_slingshot_b200.utils import lifecycle

MIB = 1 << 20


def _fixture(cycles=5, per_cycle=2, region=64 * MIB, leak_at=None, leak=0, rank=0, base=1000 * MIB):
    """`cycles` create/destroy cycles of `per_cycle` overlapping buffers; the first cycle loads
    modules (+32 MiB kept for good); `leak_at` adds `leak` bytes that are never returned."""
    recs, used, next_id = [], base, 1
    for c in range(cycles):
        if c == 0:
            used += 32 * MIB
        if leak_at is not None and c >= leak_at:
            used += leak if c == leak_at else 0
        ids = []
        for _ in range(per_cycle):
            before = used
            used += region
            recs.append({'phase': 'create', 'kind': 'Buffer', 'id': next_id, 'rank': rank, 'requested_bytes': region,
                         'alive': len(ids) + 1, 'device_used_bytes': used, 'used_before_bytes': before})
            ids.append(next_id)
            next_id += 1
        for i in ids:
            used -= region
            recs.append({'phase': 'destroy', 'kind': 'Buffer', 'id': i, 'rank': rank, 'requested_bytes': 0,
                         'alive': 0, 'device_used_bytes': used})
    return recs


def test_clean_cycles_pass():
    out = al.audit_rank(_fixture(), 0, 5)
    assert out == {'rank': 0, 'cycles': 5, 'peak_alive': 2, 'baseline_bytes': 1032 * MIB, 'max_growth_bytes': 0}


def test_growth_after_first_cycle_fails():
    with pytest.raises(ValueError, match='grows across Buffer cycles'):
        al.audit_rank(_fixture(leak_at=3, leak=16 * MIB), 0, 5)
    # within the tolerance it passes
    assert al.audit_rank(_fixture(leak_at=3, leak=2 * MIB), 0, 5)['max_growth_bytes'] == 2 * MIB


def test_unbalanced_and_missing():
    recs = _fixture()
    with pytest.raises(ValueError, match='still alive'):
        al.audit_rank(recs[:-1], 0, 5)
    with pytest.raises(ValueError, match='not created'):
        al.audit_rank(recs[1:], 0, 5)
    with pytest.raises(ValueError, match='already alive'):
        al.audit_rank([recs[0]] + recs, 0, 5)
    with pytest.raises(ValueError, match='expected 6'):
        al.audit_rank(recs, 0, 6)
    with pytest.raises(ValueError, match='no Buffer lifecycle events for rank 3'):
        al.audit_rank(recs, 3, 5)
    with pytest.raises(ValueError, match='no SymmetricRegion'):
        al.audit_rank(recs, 0, 5, kind='SymmetricRegion')


def test_record_that_measures_nothing_fails():
    recs = _fixture()
    recs[0] = dict(recs[0], device_used_bytes=recs[0]['used_before_bytes'])
    with pytest.raises(ValueError, match='requested'):
        al.audit_rank(recs, 0, 5)


def test_record_writes_jsonl_and_cli(tmp_path, monkeypatch):
    log = tmp_path / 'lifecycle-rank{rank}.jsonl'
    monkeypatch.setenv('DEEPEP_B200_LIFECYCLE_LOG', str(log))
    used = {'v': 100 * MIB}
    monkeypatch.setattr(lifecycle, 'device_used_bytes', lambda: used['v'])
    monkeypatch.setattr(lifecycle, '_alive', lifecycle.Counter())
    for _ in range(3):
        objs = [object(), object()]
        for o in objs:
            before = lifecycle.snapshot()
            used['v'] += 8 * MIB
            lifecycle.record('create', 'SymmetricRegion', o, 8 * MIB, before)
        for o in objs:
            used['v'] -= 8 * MIB
            lifecycle.record('destroy', 'SymmetricRegion', o)
    path = str(log).replace('{rank}', '0')
    recs = al.read_log(path)
    assert [r['alive'] for r in recs[:4]] == [1, 2, 1, 0]
    assert recs[0]['used_before_bytes'] == 100 * MIB and recs[0]['device_used_bytes'] == 108 * MIB
    assert al.audit_rank(recs, 0, 3, kind='SymmetricRegion')['cycles'] == 3
    assert al.main([str(log), '--cycles', '3', '--kind', 'SymmetricRegion']) == 0
    assert al.main([str(log), '--cycles', '4', '--kind', 'SymmetricRegion']) == 1
    assert al.main([str(log), '--cycles', '3', '--ranks', '2', '--kind', 'SymmetricRegion']) == 1


def test_record_is_a_no_op_when_off(tmp_path, monkeypatch):
    monkeypatch.delenv('DEEPEP_B200_LIFECYCLE_LOG', raising=False)
    monkeypatch.setattr(lifecycle, 'device_used_bytes', lambda: (_ for _ in ()).throw(AssertionError('probed')))
    assert lifecycle.snapshot() is None
    lifecycle.record('create', 'Buffer', object(), 1)
    assert list(tmp_path.iterdir()) == []


def test_multi_rank_log_files(tmp_path):
    for rank in range(2):
        with open(tmp_path / f'l{rank}.jsonl', 'w') as f:
            for r in _fixture(rank=rank):
                f.write(json.dumps(r) + '\n')
    assert al.main([str(tmp_path / 'l{rank}.jsonl'), '--ranks', '2', '--cycles', '5']) == 0
