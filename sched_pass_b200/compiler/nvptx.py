"""Compile (woven) LLVM IR for sm_100a and run it through the CUDA driver.

Code generation uses the NVPTX backend of the LLVM that llvmlite ships
(sm_100a, PTX ISA 8.7 so cluster-launch-control instructions assemble);
the resulting PTX is handed to the driver's JIT as-is. ``CudaModule`` wraps
the driver calls a fixture needs: load, look up a kernel, arm the named
control-table globals (the named-global ABI of include/sched/sched_rt.h,
what cudaMemcpyToSymbol does for a host application), launch.
"""
from __future__ import annotations

import ctypes

import llvmlite.binding as llvm
import torch

_inited = False


def _init():
    global _inited
    if not _inited:
        llvm.initialize_all_targets()
        llvm.initialize_all_asmprinters()
        _inited = True


def compile_ptx(ir_text: str, cpu: str = "sm_100a", features: str = "+ptx87", opt: int = 2) -> bytes:
    _init()
    mod = llvm.parse_assembly(ir_text)
    mod.verify()
    tm = llvm.Target.from_triple("nvptx64-nvidia-cuda").create_target_machine(cpu=cpu, features=features,
                                                                             opt=opt)
    pto = llvm.create_pipeline_tuning_options(speed_level=opt, size_level=0)
    pb = llvm.create_pass_builder(tm, pto)
    pm = pb.getModulePassManager()
    pm.run(mod, pb)
    return tm.emit_assembly(mod).encode() + b"\0"


class CudaError(RuntimeError):
    pass


# cuda.h launch-config structs, for cuLaunchKernelEx (programmatic dependent launch)
_ATTR_PROGRAMMATIC_STREAM_SERIALIZATION = 6


class _AttrValue(ctypes.Union):
    _fields_ = [("pad", ctypes.c_char * 64), ("i", ctypes.c_int)]


class _Attr(ctypes.Structure):
    _fields_ = [("id", ctypes.c_int), ("pad", ctypes.c_char * 4), ("value", _AttrValue)]


class _LaunchConfig(ctypes.Structure):
    _fields_ = [("gridDimX", ctypes.c_uint), ("gridDimY", ctypes.c_uint), ("gridDimZ", ctypes.c_uint),
                ("blockDimX", ctypes.c_uint), ("blockDimY", ctypes.c_uint), ("blockDimZ", ctypes.c_uint),
                ("sharedMemBytes", ctypes.c_uint), ("hStream", ctypes.c_void_p),
                ("attrs", ctypes.POINTER(_Attr)), ("numAttrs", ctypes.c_uint)]


class CudaModule:
    def __init__(self, ptx: bytes):
        torch.cuda.init()
        torch.zeros(1, device="cuda")  # make torch's primary context current
        self.cu = ctypes.CDLL("libcuda.so.1")
        self.mod = ctypes.c_void_p()
        self._check("cuModuleLoadData", self.cu.cuModuleLoadData(ctypes.byref(self.mod), ctypes.c_char_p(ptx)))
        self._fns = {}

    def _check(self, what, rc):
        if rc != 0:
            s = ctypes.c_char_p()
            self.cu.cuGetErrorName(rc, ctypes.byref(s))
            raise CudaError(f"{what}: {s.value.decode() if s.value else rc}")

    def function(self, name: str):
        f = self._fns.get(name)
        if f is None:
            f = ctypes.c_void_p()
            self._check("cuModuleGetFunction", self.cu.cuModuleGetFunction(ctypes.byref(f), self.mod, name.encode()))
            self._fns[name] = f
        return f

    def has_global(self, name: str) -> bool:
        d, n = ctypes.c_uint64(), ctypes.c_size_t()
        return self.cu.cuModuleGetGlobal_v2(ctypes.byref(d), ctypes.byref(n), self.mod, name.encode()) == 0

    def set_global_ptr(self, name: str, value: int) -> None:
        """Arm (value != 0) or disarm (0) a named table slot."""
        d, n = ctypes.c_uint64(), ctypes.c_size_t()
        self._check(f"cuModuleGetGlobal({name})",
                    self.cu.cuModuleGetGlobal_v2(ctypes.byref(d), ctypes.byref(n), self.mod, name.encode()))
        v = ctypes.c_uint64(value)
        torch.cuda.synchronize()
        self._check("cuMemcpyHtoD", self.cu.cuMemcpyHtoD_v2(d, ctypes.byref(v), ctypes.c_size_t(8)))

    def launch(self, name: str, grid, block, args, shared: int = 0, pdl: bool = False) -> None:
        """args: torch tensors (passed as device pointers), ints (i32),
        floats (f32) or ctypes values. ``pdl`` launches with programmatic
        stream serialization (the kernel may start while the previous grid on
        the stream drains; a woven PDL point waits for it)."""
        holders = []
        for a in args:
            if isinstance(a, torch.Tensor):
                holders.append(ctypes.c_void_p(a.data_ptr()))
            elif isinstance(a, bool) or isinstance(a, int):
                holders.append(ctypes.c_int32(int(a)))
            elif isinstance(a, float):
                holders.append(ctypes.c_float(a))
            else:
                holders.append(a)
        params = (ctypes.c_void_p * len(holders))(*[ctypes.cast(ctypes.pointer(h), ctypes.c_void_p) for h in holders])
        g = (tuple(grid) + (1, 1, 1))[:3]
        b = (tuple(block) + (1, 1, 1))[:3]
        stream = torch.cuda.current_stream().cuda_stream
        if pdl:
            attr = _Attr()
            attr.id = _ATTR_PROGRAMMATIC_STREAM_SERIALIZATION
            attr.value.i = 1
            cfg = _LaunchConfig(g[0], g[1], g[2], b[0], b[1], b[2], shared, ctypes.c_void_p(stream),
                                ctypes.pointer(attr), 1)
            self._check("cuLaunchKernelEx", self.cu.cuLaunchKernelEx(ctypes.byref(cfg), self.function(name),
                                                                     params, None))
            return
        self._check("cuLaunchKernel", self.cu.cuLaunchKernel(
            self.function(name), ctypes.c_uint(g[0]), ctypes.c_uint(g[1]), ctypes.c_uint(g[2]),
            ctypes.c_uint(b[0]), ctypes.c_uint(b[1]), ctypes.c_uint(b[2]), ctypes.c_uint(shared),
            ctypes.c_void_p(stream), params, None))

    def close(self) -> None:
        if self.mod:
            self.cu.cuModuleUnload(self.mod)
            self.mod = ctypes.c_void_p()
