"""Execute NVPTX-targeted LLVM IR on the host CPU, one simulated thread at a
time, for GPU-free checks of woven kernels.

The IR is lowered textually to host IR: the ptx_kernel convention and the
GPU address spaces are dropped, special-register intrinsics become calls to
a small harness (thread / block indices from globals the runner sets, a
monotonic counter for clock64), and hint-only inline assembly (prefetch,
discard, griddepcontrol) is removed -- those levers cannot change results,
so removing them keeps every computed value. llvmlite's MCJIT compiles the
result. Kernels that use barriers or warp collectives are outside what a
serial runner can execute.
"""
from __future__ import annotations

import ctypes
import re

import llvmlite.binding as llvm

_inited = False


def _init():
    global _inited
    if not _inited:
        llvm.initialize_native_target()
        llvm.initialize_native_asmprinter()
        _inited = True


HARNESS = r"""
@__cpu_tid = global [3 x i32] zeroinitializer
@__cpu_ctaid = global [3 x i32] zeroinitializer
@__cpu_ntid = global [3 x i32] [i32 1, i32 1, i32 1]
@__cpu_nctaid = global [3 x i32] [i32 1, i32 1, i32 1]
@__cpu_clock = global i64 1000
"""
for _reg, _arr in (("tid", "__cpu_tid"), ("ctaid", "__cpu_ctaid"), ("ntid", "__cpu_ntid"), ("nctaid", "__cpu_nctaid")):
    for _i, _ax in enumerate("xyz"):
        HARNESS += (f"define i32 @__cpu_sreg_{_reg}.{_ax}() {{\n"
                    f"  %p = getelementptr [3 x i32], ptr @{_arr}, i64 0, i64 {_i}\n"
                    f"  %v = load i32, ptr %p\n  ret i32 %v\n}}\n")
HARNESS += """define i64 @__cpu_sreg_clock64() {
  %v = load i64, ptr @__cpu_clock
  %n = add i64 %v, 13
  store i64 %n, ptr @__cpu_clock
  ret i64 %n
}
define void @__cpu_barrier() {
  ret void
}
"""


def lower_to_host(text: str) -> str:
    out = []
    for line in text.splitlines():
        s = line.strip()
        if s.startswith("target datalayout") or s.startswith("target triple"):
            continue
        if "asm sideeffect" in line and re.match(r"\s*call void asm", line):
            continue  # hint-only inline asm (prefetch / discard / PDL)
        if s.startswith("declare") and "llvm.nvvm." in s:
            continue
        line = line.replace("ptx_kernel ", "")
        line = re.sub(r"addrspacecast \(ptr addrspace\(\d+\) (@[\w.$-]+) to ptr\)", r"\1", line)
        line = re.sub(r"= addrspacecast ptr addrspace\(\d+\) (%[\w.$-]+) to ptr", r"= getelementptr i8, ptr \1, i64 0", line)
        line = re.sub(r" addrspace\(\d+\)", "", line)
        line = re.sub(r"@llvm\.nvvm\.read\.ptx\.sreg\.([\w.]+)\(\)", r"@__cpu_sreg_\1()", line)
        line = line.replace("@llvm.nvvm.barrier0()", "@__cpu_barrier()")
        out.append(line)
    return "\n".join(out) + "\n"


class HostKernel:
    """A lowered module compiled for the host. ``run(name, grid, block, args,
    argtypes)`` executes every (block, thread) serially in launch order."""

    def __init__(self, text: str):
        _init()
        host = lower_to_host(text) + HARNESS
        mod = llvm.parse_assembly(host)
        mod.triple = llvm.get_process_triple()
        mod.verify()
        tm = llvm.Target.from_default_triple().create_target_machine(opt=0)
        self.engine = llvm.create_mcjit_compiler(mod, tm)
        self.engine.finalize_object()
        self._mod = mod

    def global_addr(self, name: str) -> int:
        return self.engine.get_global_value_address(name)

    def set_global_ptr(self, name: str, value: int) -> None:
        ctypes.c_uint64.from_address(self.global_addr(name)).value = value

    def _set3(self, name, v):
        arr = (ctypes.c_int32 * 3).from_address(self.global_addr(name))
        arr[0], arr[1], arr[2] = v

    def run(self, name: str, grid, block, args, argtypes, order=None):
        fn = ctypes.CFUNCTYPE(None, *argtypes)(self.engine.get_function_address(name))
        gx, gy, gz = (tuple(grid) + (1, 1, 1))[:3]
        bx, by, bz = (tuple(block) + (1, 1, 1))[:3]
        self._set3("__cpu_nctaid", (gx, gy, gz))
        self._set3("__cpu_ntid", (bx, by, bz))
        ctas = [(x, y, z) for z in range(gz) for y in range(gy) for x in range(gx)]
        if order is not None:
            ctas = [ctas[i] for i in order]
        for cta in ctas:
            self._set3("__cpu_ctaid", cta)
            for z in range(bz):
                for y in range(by):
                    for x in range(bx):
                        self._set3("__cpu_tid", (x, y, z))
                        fn(*args)
