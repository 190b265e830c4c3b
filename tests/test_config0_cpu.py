"""The CPU-only configuration: the weaver on a paged online-softmax decode
kernel (fp32, 8 requests, 4 query heads sharing 1 KV head, head_dim 64,
page 16, lengths uniform in [16, 512], Q/K/V ~ N(0,1)), executed on the host
from its LLVM IR, against a numpy reference of the same kernel.
Pass criteria: tau = 0 bit-exact against the stock kernel; tau > 0 equal to
exact truncated softmax attention."""
import ctypes
import os
import struct

import numpy as np
import pytest

from sched_pass_b200.compiler.cpu_exec import HostKernel
from sched_pass_b200.compiler.weave import weave
from sched_pass_b200.runtime import abi

HERE = os.path.join(os.path.dirname(os.path.abspath(__file__)), "ir")
B, G, D, PS = 8, 4, 64, 16


def build(seed=0):
    rng = np.random.default_rng(seed)
    lens = rng.integers(16, 513, size=B).astype(np.int32)
    npages = ((lens + PS - 1) // PS).astype(np.int32)
    total = int(npages.sum())
    perm = rng.permutation(total).astype(np.int32)
    maxp = int(npages.max())
    bt = np.zeros((B, maxp), np.int32)
    k = 0
    for b in range(B):
        bt[b, :npages[b]] = perm[k:k + npages[b]]
        k += npages[b]
    kc = rng.standard_normal((total, PS, D)).astype(np.float32)
    vc = rng.standard_normal((total, PS, D)).astype(np.float32)
    q = rng.standard_normal((B, G, D)).astype(np.float32)
    taus = np.array([rng.integers(0, int(n) + 1) for n in lens], np.int32)
    return lens, bt, kc, vc, q, taus, maxp


def reference(lens, bt, kc, vc, q, taus=None):
    scale = 1.0 / np.sqrt(D)
    out = np.zeros((B, G, D), np.float64)
    for b in range(B):
        n = int(lens[b])
        if taus is not None and taus[b] > 0:
            n = min(n, int(taus[b]))
        pages = bt[b, :(int(lens[b]) + PS - 1) // PS]
        K = kc[pages].reshape(-1, D)[:n].astype(np.float64)
        V = vc[pages].reshape(-1, D)[:n].astype(np.float64)
        s = (K @ q[b].astype(np.float64).T).T * scale
        p = np.exp(s - s.max(-1, keepdims=True))
        out[b] = (p / p.sum(-1, keepdims=True)) @ V
    return out


class Tables:
    """Host-memory control tables in the ABI layout."""

    def __init__(self, n=64):
        self.order = np.arange(n, dtype=np.int32)
        self.ctrl = np.zeros(abi.ctrl_bytes(n), np.uint8)
        self.timer = np.zeros(n, np.uint64)

    def set_row(self, i, q=0.0, tau=0, hint=0):
        struct.pack_into("<fHB", self.ctrl, abi.CTRL_ROWS_OFF + abi.ROW_SIZE * i, q, tau, hint)

    def set_u32(self, off, v):
        struct.pack_into("<I", self.ctrl, off, v)


def run(kern, lens, bt, kc, vc, q, maxp, tables=None):
    out = np.zeros((B, G, D), np.float32)
    acc = np.zeros((B, G, D), np.float32)
    if tables is not None:
        kern.set_global_ptr("__sched_task_order", tables.order.ctypes.data)
        kern.set_global_ptr("__sched_ctrl", tables.ctrl.ctypes.data)
        kern.set_global_ptr("__sched_timer", tables.timer.ctypes.data)
    p = ctypes.c_void_p
    args = [q.ctypes.data, kc.ctypes.data, vc.ctypes.data, bt.ctypes.data, lens.ctypes.data,
            out.ctypes.data, acc.ctypes.data, maxp, G, np.log2(np.e) / np.sqrt(D)]  # log2-domain scores
    types = [p, p, p, p, p, p, p, ctypes.c_int32, ctypes.c_int32, ctypes.c_float]
    kern.run("softmax_decode", (B,), (G,), args, types)
    return out


@pytest.fixture(scope="module")
def kernels():
    src = open(os.path.join(HERE, "softmax_decode.ll")).read()
    woven, notes = weave(src)
    assert any("softmax score mask" in n for n in notes)
    return HostKernel(src), HostKernel(woven)


def test_stock_matches_numpy(kernels):
    stock, _ = kernels
    lens, bt, kc, vc, q, _, maxp = build()
    out = run(stock, lens, bt, kc, vc, q, maxp)
    ref = reference(lens, bt, kc, vc, q)
    assert np.abs(out - ref).max() < 1e-4


def test_tau0_is_bit_exact_against_stock(kernels):
    stock, woven = kernels
    lens, bt, kc, vc, q, _, maxp = build(1)
    base = run(stock, lens, bt, kc, vc, q, maxp)
    # unarmed (null slots), then armed with neutral tables, then reversed pi + timer
    assert np.array_equal(run(woven, lens, bt, kc, vc, q, maxp), base)
    t = Tables()
    assert np.array_equal(run(woven, lens, bt, kc, vc, q, maxp, t), base)
    t.order[:B] = np.arange(B - 1, -1, -1)
    t.set_u32(abi.CTRL_ORDER_SIZE_OFF, B)
    t.timer[:] = 0
    assert np.array_equal(run(woven, lens, bt, kc, vc, q, maxp, t), base)
    assert (t.timer[:B] > 0).all(), "the timer must fill every task's row"
    # timer switched off by ctrl.flags bit0: no rows written
    t.timer[:] = 0
    t.set_u32(abi.CTRL_FLAGS_OFF, abi.FLAG_TIMER_OFF)
    assert np.array_equal(run(woven, lens, bt, kc, vc, q, maxp, t), base)
    assert (t.timer == 0).all()
    # a stale order built for another launch size is ignored (identity)
    t.set_u32(abi.CTRL_ORDER_SIZE_OFF, B + 3)
    t.order[:B] = np.roll(np.arange(B), 3)
    assert np.array_equal(run(woven, lens, bt, kc, vc, q, maxp, t), base)


def test_tau_is_exact_truncated_softmax(kernels):
    _, woven = kernels
    lens, bt, kc, vc, q, taus, maxp = build(2)
    t = Tables()
    for b in range(B):
        t.set_row(b, tau=int(taus[b]))
    out = run(woven, lens, bt, kc, vc, q, maxp, t)
    ref = reference(lens, bt, kc, vc, q, taus)
    assert np.abs(out - ref).max() < 1e-4
    full = reference(lens, bt, kc, vc, q)
    cut = [b for b in range(B) if 0 < taus[b] < lens[b]]
    assert cut and all(np.abs(full[b] - ref[b]).max() > 1e-3 for b in cut)


def test_shed_quality_sweep_is_monotone(kernels):
    """Quality of the shed lever as its budget grows (the reference's tau
    sweep, test/py/eval_quality.py:31-76): tau = f * len for growing f,
    executed by the woven kernel; the cosine similarity of the output to
    full attention rises with f and reaches 1 at f = 1 (tau = len keeps
    every token: the kernel's output equals the untruncated one)."""
    _, woven = kernels
    lens, bt, kc, vc, q, _, maxp = build(3)
    full = reference(lens, bt, kc, vc, q).reshape(-1)
    cos = []
    for f in (0.1, 0.25, 0.5, 0.75, 0.9, 1.0):
        t = Tables()
        for b in range(B):
            t.set_row(b, tau=max(1, int(f * lens[b])))
        out = run(woven, lens, bt, kc, vc, q, maxp, t).reshape(-1).astype(np.float64)
        cos.append(float(out @ full / np.linalg.norm(out) / np.linalg.norm(full)))
    assert all(b > a for a, b in zip(cos, cos[1:])), cos
    assert cos[-1] > 1 - 1e-6 and cos[0] < 0.9, cos


def test_indirect_channels_word_zero_means_off():
    """Indirect channels (SCHED_TIMER_INDIRECT / SCHED_ORDER_INDIRECT, the
    reference's device channels, test/py/test_timer_indirect.py): the slot
    word holds the address of the timer rows / order table, so a controller
    retargets or switches them by rewriting one word; word 0 = timer off /
    identity order. Results stay bit-exact against stock throughout."""
    src = open(os.path.join(HERE, "softmax_decode.ll")).read()
    stock = HostKernel(src)
    woven, _ = weave(src, {"SCHED_TIMER_INDIRECT": "1", "SCHED_ORDER_INDIRECT": "1"})
    k = HostKernel(woven)
    lens, bt, kc, vc, q, _, maxp = build(6)
    base = run(stock, lens, bt, kc, vc, q, maxp)
    t = Tables()
    t.order[:B] = np.arange(B - 1, -1, -1)
    t.set_u32(abi.CTRL_ORDER_SIZE_OFF, B)
    words = np.zeros(2, np.uint64)  # [0] timer channel, [1] order channel
    k.set_global_ptr("__sched_ctrl", t.ctrl.ctypes.data)
    k.set_global_ptr("__sched_timer", words.ctypes.data)
    k.set_global_ptr("__sched_task_order", words.ctypes.data + 8)

    def launch():
        out = np.zeros((B, G, D), np.float32)
        acc = np.zeros((B, G, D), np.float32)
        p = ctypes.c_void_p
        k.run("softmax_decode", (B,), (G,),
              [q.ctypes.data, kc.ctypes.data, vc.ctypes.data, bt.ctypes.data, lens.ctypes.data, out.ctypes.data,
               acc.ctypes.data, maxp, G, np.log2(np.e) / np.sqrt(D)],
              [p, p, p, p, p, p, p, ctypes.c_int32, ctypes.c_int32, ctypes.c_float])
        return out

    # both channels off (word 0): stock behaviour, no timer rows
    assert np.array_equal(launch(), base) and (t.timer == 0).all()
    # timer channel on: every task's row fills; order still identity
    words[0] = t.timer.ctypes.data
    assert np.array_equal(launch(), base) and (t.timer[:B] > 0).all()
    # retarget the timer to a second table by rewriting the word
    other = np.zeros(64, np.uint64)
    words[0] = other.ctypes.data
    before = t.timer.copy()
    # order channel on: reversed pi, still bit-exact
    words[1] = t.order.ctypes.data
    assert np.array_equal(launch(), base)
    assert np.array_equal(t.timer, before) and (other[:B] > 0).all()
    # the order channel is live: an all-zero table sends every CTA to task 0
    t.order[:B] = 0
    out = launch()
    assert np.array_equal(out[0], base[0]) and not out[1:].any()
    words[1] = 0  # word 0: identity again
    assert np.array_equal(launch(), base)


def test_churn_steps_stay_bit_exact():
    """48 consecutive "steps" with a changing request mix (new lengths and
    pages every step), the order table rewritten each step (reversed,
    rotated, stale-sized) and the timer toggled: every step's woven output
    equals the stock kernel's (the reference's 48-step churn check,
    test/py/test_gqa_repro_steps.py)."""
    stock, woven = kernels_pair()
    t = Tables()
    for step in range(48):
        lens, bt, kc, vc, q, _, maxp = build(100 + step)
        base = run(stock, lens, bt, kc, vc, q, maxp)
        kind = step % 3
        t.order[:B] = np.arange(B - 1, -1, -1) if kind == 0 else np.roll(np.arange(B), step)
        t.set_u32(abi.CTRL_ORDER_SIZE_OFF, B if kind != 2 else B + 1)  # kind 2: stale size -> identity
        t.set_u32(abi.CTRL_FLAGS_OFF, abi.FLAG_TIMER_OFF if step % 2 else 0)
        assert np.array_equal(run(woven, lens, bt, kc, vc, q, maxp, t), base), step


_PAIR = []


def kernels_pair():
    if not _PAIR:
        src = open(os.path.join(HERE, "softmax_decode.ll")).read()
        _PAIR.extend([HostKernel(src), HostKernel(weave(src)[0])])
    return _PAIR


def test_ticket_work_queue_driver_runs_every_task():
    """The woven ticket work queue (sched-workqueue) executed on the host:
    W < B persistent workers claim tasks from the queue word (primed to W, the
    reference's host protocol) through the task order; every task runs
    (each timer row fills), results equal the stock launch of one
    CTA per task, and num_tasks = 0 takes the stock path. One thread per CTA
    (G = 1): the host runs a CTA's threads one after another, so a
    shared-memory broadcast between them cannot be emulated."""
    src = open(os.path.join(HERE, "softmax_decode.ll")).read()
    src = src.replace("@__sched_timer = ",
                      "@__sched_queue = addrspace(1) externally_initialized global ptr null, align 8\n"
                      "@__sched_timer = ")
    stock = HostKernel(src)
    woven, _ = weave(src, {"SCHED_WORKQUEUE": "1"})
    k = HostKernel(woven)
    lens, bt, kc, vc, q, _, maxp = build(9)
    q1 = np.ascontiguousarray(q[:, :1])
    p = ctypes.c_void_p
    types = [p, p, p, p, p, p, p, ctypes.c_int32, ctypes.c_int32, ctypes.c_float]

    def launch(kern, grid):
        out = np.zeros((B, 1, D), np.float32)
        acc = np.zeros((B, 1, D), np.float32)
        kern.run("softmax_decode", (grid,), (1,),
                 [q1.ctypes.data, kc.ctypes.data, vc.ctypes.data, bt.ctypes.data, lens.ctypes.data, out.ctypes.data,
                  acc.ctypes.data, maxp, 1, np.log2(np.e) / np.sqrt(D)], types)
        return out

    base = launch(stock, B)
    t = Tables()
    t.order[:B] = np.arange(B - 1, -1, -1)
    t.set_u32(abi.CTRL_ORDER_SIZE_OFF, B)
    queue = np.zeros(4, np.uint32)
    k.set_global_ptr("__sched_task_order", t.order.ctypes.data)
    k.set_global_ptr("__sched_ctrl", t.ctrl.ctypes.data)
    k.set_global_ptr("__sched_timer", t.timer.ctypes.data)
    k.set_global_ptr("__sched_queue", queue.ctypes.data)
    W = 3
    t.set_u32(abi.CTRL_NUM_TASKS_OFF, B)
    queue[0] = W
    assert np.array_equal(launch(k, W), base)
    assert (t.timer[:B] > 0).all() and (t.timer[B:] == 0).all() and queue[0] >= B
    # num_tasks = 0: the stock path (one task per CTA), still exact
    t.set_u32(abi.CTRL_NUM_TASKS_OFF, 0)
    assert np.array_equal(launch(k, B), base)
