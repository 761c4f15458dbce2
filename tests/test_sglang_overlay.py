"""SGLang overlay installer on a fabricated SGLang package tree (CPU; SGLang is not needed)."""
import hashlib
import importlib
import json
import os
import sys

import pytest

from deepep_slingshot_b200.integrations import sglang_overlay as ov

_DISPATCHER = '''
class _DeepEPDispatcherImplNormal:
    def __init__(self, async_finish=False, group=None, hidden_size=0, num_experts=0):
        self.async_finish = async_finish
        self.group = group
        self.hidden_size = hidden_size
        self.num_experts = num_experts


class DeepEPDispatcher:
    def __init__(self, normal=True, async_finish=False, **common_kwargs):
        if normal:
            self._normal_dispatcher = _DeepEPDispatcherImplNormal(
                async_finish=async_finish,
                **common_kwargs,
            )
'''


def _fake_sglang(root, dispatcher=_DISPATCHER):
    pkg = root / 'sglang'
    mod_dir = pkg / 'srt' / 'layers' / 'moe' / 'token_dispatcher'
    mod_dir.mkdir(parents=True)
    for d in [pkg, pkg / 'srt', pkg / 'srt' / 'layers', pkg / 'srt' / 'layers' / 'moe', mod_dir]:
        (d / '__init__.py').write_text('')
    (mod_dir / 'deepep.py').write_text(dispatcher)
    (pkg / 'version.py').write_text('__version__ = "0.0.test"\n')
    (pkg / '__pycache__').mkdir()
    (pkg / '__pycache__' / 'version.cpython-312.pyc').write_bytes(b'\0')
    (pkg / 'stale.pyc').write_bytes(b'\0')
    (pkg / 'version_link.py').symlink_to('version.py')
    (pkg / 'srt_link').symlink_to('srt')
    return pkg


@pytest.fixture
def clean_sglang_modules():
    saved = {k: v for k, v in sys.modules.items() if k == 'sglang' or k.startswith('sglang.')}
    yield
    for k in [k for k in sys.modules if k == 'sglang' or k.startswith('sglang.')]:
        del sys.modules[k]
    sys.modules.update(saved)


def test_overlay_copies_and_patches(tmp_path, monkeypatch, clean_sglang_modules):
    from deepep_slingshot_b200.integrations import sglang_dispatcher as sd
    src = _fake_sglang(tmp_path / 'site')
    before = {p: p.read_bytes() for p in src.rglob('*') if p.is_file() and not p.is_symlink()}
    dst = tmp_path / 'overlay' / 'sglang'
    manifest = ov.prepare_overlay(src, dst)

    # The source is untouched; caches are not copied; symlinks stay symlinks.
    assert {p: p.read_bytes() for p in src.rglob('*') if p.is_file() and not p.is_symlink()} == before
    assert not (dst / '__pycache__').exists() and not (dst / 'stale.pyc').exists()
    assert os.readlink(dst / 'version_link.py') == 'version.py'
    assert os.readlink(dst / 'srt_link') == 'srt'
    assert (dst / 'version.py').read_text() == (src / 'version.py').read_text()

    patched = (dst / ov.DISPATCHER_MODULE).read_text()
    original = (src / ov.DISPATCHER_MODULE).read_text()
    assert manifest['original_dispatcher_sha256'] == hashlib.sha256(original.encode()).hexdigest()
    assert manifest['patched_dispatcher_sha256'] == hashlib.sha256(patched.encode()).hexdigest()
    assert manifest['enable_environment'] == 'SGLANG_DEEPEP_B200=1'
    on_disk = json.loads((tmp_path / 'overlay' / ov.MANIFEST_NAME).read_text())
    assert on_disk == manifest
    assert patched.count('_DeepEPDispatcherImplNormal(') == 0 and patched.count('_class()(') == 1

    # Without the opt-in the patched module builds SGLang's own class; with it, the adapter subclass.
    sd.make_sglang_dispatcher_class.cache_clear()
    monkeypatch.syspath_prepend(str(tmp_path / 'overlay'))
    mod = importlib.import_module('sglang.srt.layers.moe.token_dispatcher.deepep')
    assert mod.__file__.startswith(str(dst))
    monkeypatch.delenv('SGLANG_DEEPEP_B200', raising=False)
    d = mod.DeepEPDispatcher(group=None, hidden_size=256, num_experts=16)
    assert type(d._normal_dispatcher) is mod._DeepEPDispatcherImplNormal
    monkeypatch.setenv('SGLANG_DEEPEP_B200', '1')
    d = mod.DeepEPDispatcher(group=None, hidden_size=256, num_experts=16)
    impl = d._normal_dispatcher
    assert isinstance(impl, mod._DeepEPDispatcherImplNormal)
    assert type(impl) is sd.make_sglang_dispatcher_class()
    assert isinstance(impl._impl, sd.DeepEPB200Normal)
    assert impl._impl.hidden_size == 256 and impl._impl.num_experts == 16
    assert impl._impl.expert_alignment == 128
    sd.make_sglang_dispatcher_class.cache_clear()


def test_overlay_refuses_existing_destination(tmp_path):
    src = _fake_sglang(tmp_path / 'site')
    dst = tmp_path / 'overlay' / 'sglang'
    dst.mkdir(parents=True)
    with pytest.raises(FileExistsError):
        ov.prepare_overlay(src, dst)
    assert list(dst.iterdir()) == []
    assert ov.main(['--source', str(src), '--destination', str(dst)]) == 1


@pytest.mark.parametrize('body', [
    _DISPATCHER.replace('self._normal_dispatcher = _DeepEPDispatcherImplNormal(', 'self._normal = make('),
    _DISPATCHER + '\n        self._normal_dispatcher = _DeepEPDispatcherImplNormal(async_finish=False)\n',
])
def test_overlay_refuses_unexpected_dispatcher(tmp_path, body):
    src = _fake_sglang(tmp_path / 'site', body)
    dst = tmp_path / 'overlay' / 'sglang'
    with pytest.raises(ValueError):
        ov.prepare_overlay(src, dst)
    assert not dst.exists() and not (tmp_path / 'overlay' / ov.MANIFEST_NAME).exists()


def test_patch_is_not_applied_twice():
    once = ov.patch_dispatcher_source(_DISPATCHER)
    with pytest.raises(ValueError):
        ov.patch_dispatcher_source(once)
    compile(once, 'deepep.py', 'exec')
