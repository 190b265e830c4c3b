"""The heterogeneous-batch fixture (tests/ir/hetero_decode.ll) woven and run
on the host: long and short requests through one kernel, the shape of the
reference's motivating experiment (jc-su/sched-pass test/hetero_batch.cu:1-20).

Checks, all against the stock kernel (one CTA per request):
* the stock kernel equals a numpy statement of the contraction;
* woven with null slots, and with a reversed task order, the output is
  bit-identical (pi changes when a request runs, never what it computes);
* the ticket work queue with W < tasks workers claiming through an LPT order
  runs every task exactly once (every timer row fills) with the same bits,
  and num_tasks = 0 takes the stock path.

One thread per CTA on the host (the work-queue claim is broadcast through
shared memory, which a serial host runner cannot emulate), so each request
computes output element 0 only."""
import ctypes
import os

import numpy as np

from sched_pass_b200.compiler.cpu_exec import HostKernel
from sched_pass_b200.compiler.weave import weave
from sched_pass_b200.runtime import abi

HERE = os.path.join(os.path.dirname(os.path.abspath(__file__)), "ir")
D, PT = 128, 64          # floats per token row, tokens per KV block
NSEQ, LONGB, SHORTB = 16, 8, 2


def _src(queue=False):
    src = open(os.path.join(HERE, "hetero_decode.ll")).read()
    if queue:
        src = src.replace("@__sched_timer = ", "@__sched_queue = addrspace(1) externally_initialized "
                                               "global ptr null, align 8\n@__sched_timer = ")
    return src


def _inputs(seed=0):
    rng = np.random.default_rng(seed)
    nbl = np.array([LONGB if t % 8 == 0 else SHORTB for t in range(NSEQ)], np.int32)
    npages = NSEQ * LONGB
    kv = rng.standard_normal(npages * PT * D).astype(np.float32)
    bt = np.array([[(t * LONGB + b * 5 + 3) % npages for b in range(LONGB)] for t in range(NSEQ)], np.int32)
    w = rng.standard_normal(PT).astype(np.float32)
    return kv, bt, nbl, w


def _launch(kern, grid, kv, bt, nbl, w, threads=1):
    out = np.zeros(NSEQ * D, np.float32)
    p = ctypes.c_void_p
    kern.run("hetero_decode", (grid,), (threads,),
             [kv.ctypes.data, bt.ctypes.data, nbl.ctypes.data, w.ctypes.data, out.ctypes.data, LONGB],
             [p, p, p, p, p, ctypes.c_int32])
    return out


class _Tables:
    def __init__(self, n=64):
        self.order = np.arange(n, dtype=np.int32)
        self.ctrl = np.zeros(abi.ctrl_bytes(n), np.uint8)
        self.timer = np.zeros(n, np.uint64)
        self.queue = np.zeros(4, np.uint32)

    def u32(self, off, v):
        np.frombuffer(self.ctrl, np.uint32, count=1, offset=off)[:] = v  # noqa: E203

    def arm(self, k, queue=False):
        k.set_global_ptr("__sched_task_order", self.order.ctypes.data)
        k.set_global_ptr("__sched_ctrl", self.ctrl.ctypes.data)
        k.set_global_ptr("__sched_timer", self.timer.ctypes.data)
        if queue:
            k.set_global_ptr("__sched_queue", self.queue.ctypes.data)


def test_stock_matches_numpy_and_woven_orders_are_bit_exact():
    kv, bt, nbl, w = _inputs(1)
    stock = HostKernel(_src())
    base = _launch(stock, NSEQ, kv, bt, nbl, w, threads=4)
    kv3 = kv.reshape(-1, PT, D)
    for r in range(NSEQ):
        ref = sum((kv3[bt[r, b]] * w[:, None]).sum(0, dtype=np.float64) for b in range(nbl[r]))
        assert np.allclose(base.reshape(NSEQ, D)[r, :4], ref[:4], rtol=1e-4, atol=1e-4)
    woven = HostKernel(weave(_src(), {})[0])
    assert np.array_equal(_launch(woven, NSEQ, kv, bt, nbl, w, threads=4), base)  # null slots
    t = _Tables()
    t.order[:NSEQ] = np.arange(NSEQ - 1, -1, -1)
    t.u32(abi.CTRL_ORDER_SIZE_OFF, NSEQ)
    t.arm(woven)
    assert np.array_equal(_launch(woven, NSEQ, kv, bt, nbl, w, threads=4), base)  # reversed pi
    assert (t.timer[:NSEQ] > 0).all()


def test_ticket_workers_claim_every_request_in_lpt_order():
    kv, bt, nbl, w = _inputs(2)
    base = _launch(HostKernel(_src(queue=True)), NSEQ, kv, bt, nbl, w)
    k = HostKernel(weave(_src(queue=True), {"SCHED_WORKQUEUE": "1"})[0])
    t = _Tables()
    t.order[:NSEQ] = np.argsort(-nbl, kind="stable")  # longest first
    t.u32(abi.CTRL_ORDER_SIZE_OFF, NSEQ)
    t.u32(abi.CTRL_NUM_TASKS_OFF, NSEQ)
    t.arm(k, queue=True)
    W = 4
    t.queue[0] = W  # the ticket is primed to the worker count
    assert np.array_equal(_launch(k, W, kv, bt, nbl, w), base)
    assert (t.timer[:NSEQ] > 0).all() and int(t.queue[0]) >= NSEQ
    t.u32(abi.CTRL_NUM_TASKS_OFF, 0)  # disarm switch: stock path, one task per CTA
    assert np.array_equal(_launch(k, NSEQ, kv, bt, nbl, w), base)
