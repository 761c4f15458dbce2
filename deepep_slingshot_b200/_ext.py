"""Loader of the in-tree sm_100a extension `deepep_slingshot_b200._C`.

The extension is required on a GPU: there is no silent fallback. On a CPU-only machine the package
still imports (the reference backend and host-side utilities work without it), and
`require_ext()` raises with the build command.
"""
import importlib

_ext = None
_err = None


def load_ext():
    """The in-tree extension module, or None when it is not built (the error is kept for `require_ext`)."""
    global _ext, _err
    if _ext is None and _err is None:
        try:
            _ext = importlib.import_module('deepep_slingshot_b200._C')
        except ImportError as e:  # not built yet
            _err = e
    return _ext


def require_ext():
    """The in-tree extension module; raises with the build command when it is not built."""
    ext = load_ext()
    if ext is None:
        raise RuntimeError('deepep_slingshot_b200._C is not built: run `python setup.py build_ext --inplace` '
                           f'at the repository root (import error: {_err})')
    return ext
