"""Make an SGLang overlay whose normal-mode DeepEP dispatcher can be switched to this library.

    python -m deepep_slingshot_b200.integrations.sglang_overlay \
        --source <site-packages>/sglang --destination <new dir>/sglang

The reference's installer (backend/tools/prepare_sglang_overlay.py) copies the inspected SGLang
package into a new directory and patches an environment opt-in into the dispatcher constructor; an
existing installation is never modified. This installer keeps those rules:

  * the destination must not exist; the source is only read;
  * the package is copied file by file (contents only: no modes, owners or extended attributes),
    symlinks stay symlinks, `__pycache__` and `.pyc` files are skipped;
  * `srt/layers/moe/token_dispatcher/deepep.py` must contain exactly one construction of
    `_DeepEPDispatcherImplNormal` assigned to `self._normal_dispatcher`; anything else stops the
    installer before it writes a file (the SGLang version differs from the one this was written for);
  * the construction is routed through a selector appended to that module: with
    `SGLANG_DEEPEP_B200=1` in the environment it builds
    `integrations.sglang_dispatcher.make_sglang_dispatcher_class()`, otherwise SGLang's own class;
  * a manifest (`deepep-b200-sglang-manifest.json`, beside the destination) records the source,
    the SHA-256 of the original and patched modules and of the adapter, and the opt-in variable.

The adapter is imported from this package (which must be importable where SGLang runs), so the
overlay holds no copy of it.
"""
import argparse
import hashlib
import json
import os
import re
import shutil
import sys
from pathlib import Path
from typing import Dict

DISPATCHER_MODULE = Path('srt/layers/moe/token_dispatcher/deepep.py')
ENABLE_ENV = 'SGLANG_DEEPEP_B200'
MANIFEST_NAME = 'deepep-b200-sglang-manifest.json'

# `self._normal_dispatcher = _DeepEPDispatcherImplNormal(` at any indentation.
_CONSTRUCTION = re.compile(r'^([ \t]*self\._normal_dispatcher[ \t]*=[ \t]*)_DeepEPDispatcherImplNormal\(', re.M)
_SELECTOR_NAME = '_deepep_b200_normal_dispatcher_class'
_SELECTOR = f'''

def {_SELECTOR_NAME}():
    """Normal-mode dispatcher class: the DeepEP B200 adapter when {ENABLE_ENV}=1, else SGLang's own."""
    import os
    if os.getenv("{ENABLE_ENV}") == "1":
        from deepep_slingshot_b200.integrations.sglang_dispatcher import make_sglang_dispatcher_class
        return make_sglang_dispatcher_class()
    return _DeepEPDispatcherImplNormal
'''


def _sha256(data: bytes) -> str:
    return hashlib.sha256(data).hexdigest()


def patch_dispatcher_source(text: str) -> str:
    """The dispatcher module with its normal-mode construction routed through the selector.
    Raises ValueError unless the construction occurs exactly once and the module is unpatched."""
    if _SELECTOR_NAME in text:
        raise ValueError('the dispatcher module is already patched')
    found = _CONSTRUCTION.findall(text)
    if len(found) != 1:
        raise ValueError(f'expected one normal-mode dispatcher construction, found {len(found)}; '
                         'review this SGLang version before adapting the installer')
    patched = _CONSTRUCTION.sub(lambda m: m.group(1) + f'{_SELECTOR_NAME}()(', text, count=1)
    return patched.rstrip('\n') + '\n' + _SELECTOR


def _copy_tree(source: Path, destination: Path) -> int:
    """Copy file contents under `source` into the new `destination`; returns the number of entries."""
    count = 0
    for directory, subdirs, files in os.walk(source, followlinks=False):
        subdirs[:] = [d for d in subdirs if d != '__pycache__']
        rel = Path(directory).relative_to(source)
        target = destination / rel
        target.mkdir(parents=True, exist_ok=True)
        for name in list(subdirs):
            src = Path(directory) / name
            if src.is_symlink():
                (target / name).symlink_to(os.readlink(src))
                subdirs.remove(name)
                count += 1
        for name in files:
            if name.endswith('.pyc'):
                continue
            src = Path(directory) / name
            if src.is_symlink():
                (target / name).symlink_to(os.readlink(src))
            else:
                shutil.copyfile(src, target / name)
            count += 1
    return count


def prepare_overlay(source: Path, destination: Path) -> Dict[str, str]:
    """Copy `source` (an SGLang package directory) to the new `destination` and patch the opt-in.
    Returns the manifest, which is also written beside `destination`."""
    source, destination = Path(source).resolve(), Path(destination).absolute()
    if destination.exists() or destination.is_symlink():
        raise FileExistsError(f'{destination} exists: an overlay is always made in a new directory')
    module_src = source / DISPATCHER_MODULE
    original = module_src.read_text()
    patched = patch_dispatcher_source(original)  # fails before anything is written
    destination.mkdir(parents=True)
    entries = _copy_tree(source, destination)
    module_dst = destination / DISPATCHER_MODULE
    module_dst.write_text(patched)
    from . import sglang_dispatcher
    adapter = Path(sglang_dispatcher.__file__)
    manifest = {
        'source_root': str(source),
        'destination': str(destination),
        'copied_entries': str(entries),
        'original_dispatcher_sha256': _sha256(original.encode()),
        'patched_dispatcher_sha256': _sha256(module_dst.read_bytes()),
        'adapter_module': str(adapter),
        'adapter_sha256': _sha256(adapter.read_bytes()),
        'enable_environment': f'{ENABLE_ENV}=1',
    }
    (destination.parent / MANIFEST_NAME).write_text(json.dumps(manifest, indent=2) + '\n')
    return manifest


def main(argv=None) -> int:
    p = argparse.ArgumentParser(description=__doc__.split('\n')[0])
    p.add_argument('--source', type=Path, required=True, help='the installed sglang package directory')
    p.add_argument('--destination', type=Path, required=True, help='new directory for the overlay package')
    args = p.parse_args(argv)
    try:
        manifest = prepare_overlay(args.source, args.destination)
    except (FileExistsError, FileNotFoundError, ValueError) as e:
        print(f'overlay not made: {e}', file=sys.stderr)
        return 1
    print(json.dumps(manifest, indent=2))
    return 0


if __name__ == '__main__':
    sys.exit(main())
