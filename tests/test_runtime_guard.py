"""NCCL runtime guard: synthetic `/proc/self/maps` text over real temporary library files (CPU)."""
import pytest

from deepep_slingshot_b200.utils import runtime_guard as rg


def _maps(*paths):
    return ''.join(f'7f0000000000-7f0000001000 r-xp 00000000 00:01 {i} {p}\n' for i, p in enumerate(paths))


@pytest.fixture
def libs(tmp_path, monkeypatch):
    monkeypatch.delenv('DEEPEP_B200_SUPPRESS_NCCL_CHECK', raising=False)
    (tmp_path / 'wheel').mkdir()
    (tmp_path / 'system').mkdir()
    (tmp_path / 'copy').mkdir()
    wheel = tmp_path / 'wheel' / 'libnccl.so.2'
    wheel.write_bytes(b'runtime-2.28')
    system = tmp_path / 'system' / 'libnccl.so.2.27.3'
    system.write_bytes(b'runtime-2.27')
    copy = tmp_path / 'copy' / 'libnccl.so.2'
    copy.write_bytes(b'runtime-2.28')
    link = tmp_path / 'system' / 'libnccl.so'
    link.symlink_to(wheel)
    return {'wheel': str(wheel), 'system': str(system), 'copy': str(copy), 'link': str(link),
            'net': str(tmp_path / 'wheel' / 'libnccl-net.so'), 'tuner': str(tmp_path / 'libnccl-tuner-ofi.so')}


def test_one_runtime_mapped_many_times(libs):
    maps = _maps(libs['wheel'], libs['wheel'], libs['wheel'])
    assert rg.mapped_nccl_runtimes(maps) == [libs['wheel']]
    assert rg.check_nccl_runtime(maps, expected=libs['wheel']) == libs['wheel']


def test_plugins_are_not_runtimes(libs):
    maps = _maps(libs['net'], libs['wheel'], libs['tuner'])
    assert rg.mapped_nccl_runtimes(maps) == [libs['wheel']]
    assert rg.check_nccl_runtime(maps, expected=libs['wheel']) == libs['wheel']
    assert rg.check_nccl_runtime(_maps(libs['net'], libs['tuner']), expected=libs['wheel']) is None


def test_two_different_runtimes_rejected(libs):
    with pytest.raises(rg.NcclRuntimeError, match='two NCCL runtimes'):
        rg.check_nccl_runtime(_maps(libs['wheel'], libs['system']), expected=None)


def test_same_library_through_two_paths_accepted(libs):
    assert rg.check_nccl_runtime(_maps(libs['wheel'], libs['link']), expected=libs['wheel']) == libs['wheel']
    assert rg.check_nccl_runtime(_maps(libs['wheel'], libs['copy']), expected=libs['copy']) == libs['wheel']


def test_unexpected_runtime_rejected(libs):
    with pytest.raises(rg.NcclRuntimeError, match='not the one PyTorch ships'):
        rg.check_nccl_runtime(_maps(libs['system']), expected=libs['wheel'])


def test_deleted_mapping_and_short_lines(libs):
    maps = _maps(libs['wheel']) + '7f00-7f01 rw-p 00000000 00:00 0\n' + \
        f'7f02-7f03 r-xp 00000000 00:01 9 {libs["system"]} (deleted)\n'
    assert rg.mapped_nccl_runtimes(maps) == [libs['wheel'], libs['system']]


def test_suppressed(libs, monkeypatch):
    monkeypatch.setenv('DEEPEP_B200_SUPPRESS_NCCL_CHECK', '1')
    assert rg.check_nccl_runtime(_maps(libs['wheel'], libs['system'])) is None


def test_this_process_passes(monkeypatch):
    """torch (already imported by the test session) maps at most the runtime its wheel ships."""
    monkeypatch.delenv('DEEPEP_B200_SUPPRESS_NCCL_CHECK', raising=False)
    import torch  # noqa: F401
    import torch.distributed  # noqa: F401
    mapped = rg.check_nccl_runtime()
    expected = rg.expected_nccl_runtime()
    if mapped is not None and expected is not None:
        assert rg._same_library(mapped, expected)
