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

# bindings that launch kernels, with the number of kernel launches per call
LAUNCHERS = {
    "gemm": 1, "gemm_qkv_rope": 1, "gemm_allreduce": 1, "gemm_reduce_scatter": 1, "sp_reduce_norm": 1,
    "sp_wait_rows": 1, "attn_decode": 1, "attn_merge": 1, "attn_prefill": 1, "add_rmsnorm": 1,
    "rope_kv_append": 1, "embedding": 1, "argmax": 1, "argmax_exchange": 1, "moe_router": 1, "kv_page_copy": 1,
    "kv_page_copy_fp8": 1, "moe_dispatch": 1, "moe_expert_gemm": 1, "moe_quantize": 1,
    "moe_combine_norm": 1, "probe_stream": 1, "probe_tasks": 1, "probe_mix": 1, "probe_clc": 1, "probe_clc_shape": 1, "probe_pdl_pairs": 2,
    "probe_pdl_produce": 1,
}


class _Counted:
    """The extension module with a count of the kernel launches its
    launchers issued (``launches``). A call issued while a CUDA graph is being
    captured is counted once, at capture; callers that replay graphs add the
    graph's count per replay (``Engine``)."""

    def __init__(self, mod):
        self._mod = mod
        self.launches = 0

    def __getattr__(self, name):
        f = getattr(self._mod, name)
        n = LAUNCHERS.get(name)
        if n is None or not callable(f):
            return f

        take = self._mod.take_error

        def counted(*a, **k):
            self.launches += n
            r = f(*a, **k)
            rc, op = take()  # launch errors are recorded by the binding, raised here
            if rc:
                raise RuntimeError(f"{op} launch failed (code {rc})")
            return r

        counted.__name__ = name
        self.__dict__[name] = counted  # later lookups skip __getattr__
        return counted


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
            _mod = _Counted(_build.build_extension())
            return _mod
        if _build.EXT_NAME in sys.modules:
            _mod = _Counted(sys.modules[_build.EXT_NAME])
            return _mod
        spec = importlib.util.spec_from_file_location(_build.EXT_NAME, path)
        if spec is None or spec.loader is None:
            raise ImportError(f"cannot load native extension at {path}")
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
        sys.modules[_build.EXT_NAME] = mod
        _mod = _Counted(mod)
        return _mod


def ext_loaded() -> bool:
    return _mod is not None


def launches() -> int:
    """Kernel launches issued through the extension so far in this process."""
    return _mod.launches if _mod is not None else 0
