"""Null slots stay bit-exact, for every fixture and every lever-knob
combination: each woven variant verifies under LLVM and, executed on the
host with no control tables installed, computes exactly what the stock
kernel computes (the contract that a disarmed weave is inert); armed with
neutral tables it is still exact, and the timer fills its rows exactly when
it is compiled in."""
import ctypes
import itertools
import os

import numpy as np
import pytest

from sched_pass_b200.compiler.cpu_exec import HostKernel
from sched_pass_b200.compiler.weave import weave
from sched_pass_b200.runtime import abi

HERE = os.path.join(os.path.dirname(os.path.abspath(__file__)), "ir")
KNOBS = ["SCHED_NO_INDIRECT", "SCHED_NO_SHED", "SCHED_NO_POLICY", "SCHED_NO_TIMER", "SCHED_PDL"]
P = ctypes.c_void_p


def case_softmax_decode(rng):
    B, G, D, PS = 4, 2, 64, 16
    lens = rng.integers(16, 100, size=B).astype(np.int32)
    maxp = int(((lens + PS - 1) // PS).max())
    bt = rng.permutation(B * maxp).astype(np.int32).reshape(B, maxp)
    kc = rng.standard_normal((B * maxp, PS, D)).astype(np.float32)
    vc = rng.standard_normal((B * maxp, PS, D)).astype(np.float32)
    q = rng.standard_normal((B, G, D)).astype(np.float32)

    def run(k):
        out, acc = np.zeros((B, G, D), np.float32), np.zeros((B, G, D), np.float32)
        k.run("softmax_decode", (B,), (G,), [q.ctypes.data, kc.ctypes.data, vc.ctypes.data, bt.ctypes.data,
                                              lens.ctypes.data, out.ctypes.data, acc.ctypes.data, maxp, G, 0.18],
              [P] * 7 + [ctypes.c_int32, ctypes.c_int32, ctypes.c_float])
        return out
    return run


def case_paged_linear(rng):
    R, NB, D = 5, 6, 64
    kv = rng.standard_normal((R * NB, 64)).astype(np.float32)
    bt = rng.permutation(R * NB).astype(np.int32)
    w = rng.standard_normal(NB).astype(np.float32)

    def run(k):
        out = np.zeros((R, D), np.float32)
        k.run("paged_linear", (R,), (D,), [kv.ctypes.data, bt.ctypes.data, w.ctypes.data, out.ctypes.data, NB],
              [P, P, P, P, ctypes.c_int32])
        return out
    return run


def case_arith_decode(rng):
    R, NT, D = 4, 12, 64
    kv = rng.standard_normal((R * NT, D)).astype(np.float32)
    w = rng.standard_normal(NT).astype(np.float32)

    def run(k):
        out = np.zeros((R, D), np.float32)
        k.run("arith_decode", (R,), (D,), [kv.ctypes.data, w.ctypes.data, out.ctypes.data, NT],
              [P, P, P, ctypes.c_int32])
        return out
    return run


CASES = {"softmax_decode.ll": case_softmax_decode, "paged_linear.ll": case_paged_linear,
         "arith_decode.ll": case_arith_decode}


@pytest.mark.parametrize("fixture", sorted(CASES))
def test_every_knob_combination_is_inert_when_disarmed(fixture):
    src = open(os.path.join(HERE, fixture)).read()
    run = CASES[fixture](np.random.default_rng(0))
    base = run(HostKernel(src))
    import llvmlite.binding as llvm
    llvm.initialize_all_targets()
    llvm.initialize_all_asmprinters()
    for r in range(len(KNOBS) + 1):
        for combo in itertools.combinations(KNOBS, r):
            out, _ = weave(src, {k: "1" for k in combo})
            llvm.parse_assembly(out).verify()
            k = HostKernel(out)
            assert np.array_equal(run(k), base), (fixture, combo)
            # armed with neutral tables: identity order, tau 0, q 0, hint auto, timer on
            order = np.arange(4096, dtype=np.int32)
            ctrl = np.zeros(abi.ctrl_bytes(4096), np.uint8)
            timer = np.zeros(4096, np.uint64)
            k.set_global_ptr("__sched_task_order", order.ctypes.data)
            k.set_global_ptr("__sched_ctrl", ctrl.ctypes.data)
            k.set_global_ptr("__sched_timer", timer.ctypes.data)
            assert np.array_equal(run(k), base), (fixture, combo, "neutral tables")
            assert ("SCHED_NO_TIMER" in combo) == (not timer.any()), (fixture, combo)
