"""Read-only GPU health snapshot (`utils/gpu_health.py`) against a fake NVML, and the ladder's
resume gate on it (CPU)."""
from deepep_slingshot_b200.utils import gpu_health


class FakeNvml:
    def __init__(self, gpus):
        self.gpus = gpus  # list of dicts
        self.calls = []

    def nvmlDeviceGetCount(self):
        return len(self.gpus)

    def nvmlDeviceGetHandleByIndex(self, i):
        return i

    def nvmlDeviceGetName(self, h):
        return b'NVIDIA B200'

    def nvmlDeviceGetTemperature(self, h, sensor):
        return self.gpus[h].get('temp', 40)

    def nvmlDeviceGetTotalEccErrors(self, h, err_type, counter):
        if 'ecc' not in self.gpus[h]:
            raise RuntimeError('not supported')
        assert (err_type, counter) == (1, 0)
        return self.gpus[h]['ecc']

    def nvmlDeviceGetRetiredPagesPendingStatus(self, h):
        return self.gpus[h].get('retire', 0)

    def nvmlDeviceGetRemappedRows(self, h):
        return (0, 0, self.gpus[h].get('remap', 0), 0)

    def nvmlDeviceGetCurrentClocksEventReasons(self, h):
        return self.gpus[h].get('reasons', 0)


def test_snapshot_flags_device_problems():
    nv = FakeNvml([{'ecc': 0}, {'ecc': 3, 'reasons': gpu_health.HW_SLOWDOWN | 0x4}, {'remap': 1},
                   {'reasons': gpu_health.SW_THERMAL_SLOWDOWN}])
    rep = gpu_health.snapshot(nv)
    assert [g.index for g in rep] == [0, 1, 2, 3]
    assert rep[0].problems == [] and rep[0].name == 'NVIDIA B200' and rep[0].temperature_c == 40
    assert rep[1].problems == ['3 uncorrected ECC errors', 'hw_slowdown active']   # 0x4 (power cap) is not a problem
    assert rep[2].problems == ['row remapping pending']
    assert rep[3].uncorrected_ecc is None and rep[3].problems == ['sw_thermal_slowdown active']
    lines = gpu_health.unhealthy(rep)
    assert len(lines) == 3 and lines[0].startswith('GPU 1 (NVIDIA B200)')


def test_snapshot_only_queries():
    import inspect
    src = inspect.getsource(gpu_health)
    for setter in ('nvmlDeviceSet', 'nvmlDeviceReset', 'nvmlDeviceClear', 'nvmlDeviceSetPersistenceMode'):
        assert setter + '(' not in src


def test_ladder_resume_needs_a_clean_health_check(tmp_path):
    from deepep_slingshot_b200.harness.ladder import load_state, run_ladder
    gates = [{'name': 'a', 'args': []}, {'name': 'b', 'args': []}]
    fail = {'b': True}

    def fake(gate, d):
        return ['boom'] if fail.get(gate['name']) else []
    out = str(tmp_path)
    assert not run_ladder(out, fake, gates)
    fail['b'] = False
    assert not run_ladder(out, fake, gates, resume_reason='fixed', health_check=lambda: ['GPU 0: hw_slowdown active'])
    assert load_state(tmp_path / 'ladder_state.json')['failed'] == 'b'   # still stopped
    assert run_ladder(out, fake, gates, resume_reason='fixed', health_check=lambda: [])
    st = load_state(tmp_path / 'ladder_state.json')
    assert st['passed'] == ['a', 'b'] and st['resumes'][-1]['health_checked'] is True
