"""Loading of the native kernel extension.

The kernels exist only as sm_100a CUDA code: there is no Python or library
fallback for them. ``ext()`` imports the in-tree build (compiling it first if
the shared object is missing) and raises if that fails, so a GPU run can
never silently take a non-native path.
"""
from __future__ import annotations

import importlib.util
import os
import sys
import threading

from . import _build

_lock = threading.Lock()
_mod = None


def ext():
    global _mod
    if _mod is not None:
        return _mod
    with _lock:
        if _mod is not None:
            return _mod
        import torch  # noqa: F401  (the extension links against libtorch)

        path = _build.ext_path()
        if os.environ.get("SCHED_B200_REBUILD") == "1" or not os.path.exists(path):
            _mod = _build.build_extension()
            return _mod
        if _build.EXT_NAME in sys.modules:
            _mod = sys.modules[_build.EXT_NAME]
            return _mod
        spec = importlib.util.spec_from_file_location(_build.EXT_NAME, path)
        if spec is None or spec.loader is None:
            raise ImportError(f"cannot load native extension at {path}")
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
        sys.modules[_build.EXT_NAME] = mod
        _mod = mod
        return _mod


def ext_loaded() -> bool:
    return _mod is not None
