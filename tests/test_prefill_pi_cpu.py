"""Task-order and timer levers on a causal paged *prefill* kernel (the
reference weaves FlashInfer's prefill with pi + timer,
test/py/test_flashinfer_prefill.py): the woven fixture runs on the host on a
2-D grid (query tiles x heads, pi on the tile axis); stock, disarmed,
reversed and LPT orders give the same bits, every tile's timer row fills,
and the per-request fold of the tile rows accounts for every tile of a
request that was prefilled in several tiles."""
import ctypes
import os
import struct

import numpy as np
import pytest

from sched_pass_b200.compiler.cpu_exec import HostKernel
from sched_pass_b200.compiler.weave import weave
from sched_pass_b200.runtime import abi

HERE = os.path.join(os.path.dirname(os.path.abspath(__file__)), "ir")
HQ, G, D, PS, ROWS = 4, 2, 64, 16, 16
HKV = HQ // G


def build(seed=0):
    """Three prefill segments: (request, first position, rows) -- the second
    continues a prompt whose first 64 tokens are already cached."""
    rng = np.random.default_rng(seed)
    segs = [(0, 0, 70), (1, 64, 90), (2, 0, 37)]
    ctx = [s + n for _, s, n in segs]
    maxp = max((c + PS - 1) // PS for c in ctx)
    total = sum((c + PS - 1) // PS for c in ctx)
    perm = rng.permutation(total).astype(np.int32)
    bt = np.zeros((3, maxp), np.int32)
    k = 0
    for r, c in enumerate(ctx):
        npg = (c + PS - 1) // PS
        bt[r, :npg] = perm[k:k + npg]
        k += npg
    kc = rng.standard_normal((total, HKV, PS, D)).astype(np.float32)
    vc = rng.standard_normal((total, HKV, PS, D)).astype(np.float32)
    nrows = sum(n for _, _, n in segs)
    q = rng.standard_normal((nrows, HQ, D)).astype(np.float32)
    tiles, row = [], 0
    for r, s, n in segs:
        for t0 in range(0, n, ROWS):
            tiles.append((r, row + t0, min(ROWS, n - t0), s + t0))
        row += n
    return segs, bt, kc, vc, q, np.array(tiles, np.int32), maxp


def reference(segs, bt, kc, vc, q):
    out = np.zeros_like(q, dtype=np.float64)
    row = 0
    for r, s, n in segs:
        pages = bt[r]
        for i in range(n):
            p = s + i
            for h in range(HQ):
                K = kc[pages][:, h // G].reshape(-1, D)[:p + 1].astype(np.float64)
                V = vc[pages][:, h // G].reshape(-1, D)[:p + 1].astype(np.float64)
                sc = K @ q[row + i, h].astype(np.float64) / np.sqrt(D)
                w = np.exp(sc - sc.max())
                out[row + i, h] = (w / w.sum()) @ V
        row += n
    return out


def launch(k, case, tables=None):
    segs, bt, kc, vc, q, tiles, maxp = case
    out = np.zeros_like(q)
    acc = np.zeros_like(q)
    if tables is not None:
        order, ctrl, timer = tables
        k.set_global_ptr("__sched_task_order", order.ctypes.data)
        k.set_global_ptr("__sched_ctrl", ctrl.ctypes.data)
        k.set_global_ptr("__sched_timer", timer.ctypes.data)
    p = ctypes.c_void_p
    k.run("softmax_prefill", (len(tiles), HQ), (ROWS,),
          [q.ctypes.data, kc.ctypes.data, vc.ctypes.data, bt.ctypes.data, tiles.ctypes.data, out.ctypes.data,
           acc.ctypes.data, maxp, G, HQ, np.log2(np.e) / np.sqrt(D)],
          [p, p, p, p, p, p, p, ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, ctypes.c_float])
    return out


@pytest.fixture(scope="module")
def kernels():
    src = open(os.path.join(HERE, "softmax_prefill.ll")).read()
    woven, notes = weave(src)
    assert any("remapped 1 ctaid" in n for n in notes)
    return HostKernel(src), HostKernel(woven)


def tables(order, n):
    ctrl = np.zeros(abi.ctrl_bytes(64), np.uint8)
    struct.pack_into("<I", ctrl, abi.CTRL_ORDER_SIZE_OFF, n)
    o = np.arange(64, dtype=np.int32)
    o[:n] = order
    return o, ctrl, np.zeros(64, np.uint64)


def test_prefill_levers_bit_exact_and_timer_fold(kernels):
    stock, woven = kernels
    case = build(1)
    segs, *_rest = case
    tiles = case[5]
    n = len(tiles)
    base = launch(stock, case)
    assert np.abs(base - reference(*case[:5])).max() < 1e-4
    assert np.array_equal(launch(woven, case), base)  # null slots: stock
    rev = tables(np.arange(n - 1, -1, -1), n)
    assert np.array_equal(launch(woven, case, rev), base)
    timer = rev[2]
    assert (timer[:n] > 0).all() and (timer[n:] == 0).all()
    # LPT by the causal cost of a tile (rows x keys), longest first
    cost = tiles[:, 2].astype(np.int64) * (tiles[:, 3] + tiles[:, 2])
    lpt = tables(np.argsort(-cost, kind="stable"), n)
    assert np.array_equal(launch(woven, case, lpt), base)
    # per-request fold of the tile rows (a request split over tiles sums them)
    fold = np.bincount(tiles[:, 0], weights=lpt[2][:n].astype(np.float64), minlength=3)
    per_tile = lpt[2][:n].astype(np.float64)
    for r in range(3):
        assert fold[r] == per_tile[tiles[:, 0] == r].sum() > 0
    assert (np.bincount(tiles[:, 0]) == [5, 6, 3]).all()
