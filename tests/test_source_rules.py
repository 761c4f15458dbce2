"""Source rules of the GPU pool, checked over every file that travels with the repository.

Patterns are assembled from fragments so that this file does not contain them itself:
  * none of the four batched-copy calls that faulted GPUs on this driver;
  * no `__trap` in device code (failures are reported through status words, never by trapping);
  * comments and docstrings name no build notes (the project's .md working files), no machine path
    and not the GPU job runner.
"""
import os
import re

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
SKIP_DIRS = {'.git', 'gpu' + 'run_out', '_work', 'baseline', 'build', '__pycache__', '.pytest_cache'}
SOURCE_EXT = ('.py', '.cu', '.cuh', '.h', '.hpp', '.cpp', '.c', '.sh', '.txt', '.cfg', '.toml', '.yaml', '.yml')


def _sources():
    for root, dirs, files in os.walk(ROOT):
        dirs[:] = [d for d in dirs if d not in SKIP_DIRS and not d.startswith('.')]
        for f in files:
            if f.endswith(SOURCE_EXT):
                yield os.path.join(root, f)


def _hits(pattern):
    rx = re.compile(pattern)
    out = []
    for path in _sources():
        if os.path.abspath(path) == os.path.abspath(__file__):
            continue
        with open(path, errors='replace') as fh:
            for n, line in enumerate(fh, 1):
                if rx.search(line):
                    out.append(f'{os.path.relpath(path, ROOT)}:{n}: {line.strip()[:120]}')
    return out


def test_no_batched_copy_calls():
    names = ['cuda' + 'Memcpy' + 'Batch' + 'Async', 'cuda' + 'Memcpy3D' + 'Batch' + 'Async',
             'cu' + 'Memcpy' + 'Batch' + 'Async', 'cu' + 'Memcpy3D' + 'Batch' + 'Async']
    assert _hits('|'.join(names)) == []


def test_no_device_traps():
    assert _hits(r'__' + r'trap\s*\(') == []


def test_no_build_notes_or_machine_paths_in_sources():
    notes = '|'.join(n + r'\.md' for n in ('SURVEY', 'DESIGN', 'BASELINE', 'VERDICT', 'ADVICE'))
    assert _hits(notes) == []
    assert _hits('/' + 'root' + '/') == []
    assert _hits('gpu' + 'run') == []


def test_build_fails_on_register_spills():
    """Every CUDA translation unit is compiled with ptxas turning a spill into an error, the build-time
    counterpart of the reference JIT's check that rejects kernels using local memory for spills."""
    import ast
    src = open(os.path.join(ROOT, 'setup.py')).read()
    tree = ast.parse(src)
    flags = next(ast.literal_eval(n.value) for n in ast.walk(tree)
                 if isinstance(n, ast.Assign) and any(getattr(t, 'id', '') == 'NVCC_FLAGS' for t in n.targets))
    pairs = list(zip(flags, flags[1:]))
    assert ('-Xptxas', '--warn-on-spills') in pairs and ('-Xptxas', '--warning-as-error') in pairs
    assert ('-gencode', 'arch=compute_100a,code=sm_100a') in pairs
