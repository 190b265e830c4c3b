"""Heterogeneous continuous batch on B200: the reference's motivating
experiment (jc-su/sched-pass test/hetero_batch.cu, README.md:137) on this
framework's weaver and work-queue driver.

64 requests -- 8 long (32 KV blocks) and 56 short (4 blocks), every 8th one
long -- run through ``tests/ir/hetero_decode.ll`` (one CTA per request,
128 threads, blocks of 64 tokens x 128 fp32). The step time is the makespan
of the launch. Arms, every one checked bit for bit against the stock launch:

* ``static``      stock kernel, grid = 64 (one CTA per request, no claims);
* ``identity``    ticket work queue, W = 16 persistent workers, identity order;
* ``segregated``  shorts first, longs last (the adversarial list order);
* ``lpt``         order by the woven timer's measured cycles, descending
                  (one profiling step first: the closed loop);
* ``lpt_hints``   LPT plus L2 hints: long requests POLITE (evict_first
                  streams), short ones URGENT (evict_last);
* ``clc``         cluster-launch-control work queue (grid = 64), LPT order.

The reference measured 405 -> 272 -> 265 us/step for identity -> LPT ->
LPT + hints on an RTX A6000 (sm_86); here the same arms run on one B200.

    python -m sched_pass_b200.benchmarks.hetero_batch [--iters 100]
"""
from __future__ import annotations

import argparse
import json
import os

import numpy as np
import torch

from ..runtime import abi

HERE = os.path.join(os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))), "tests", "ir")
D, PT = 128, 64
HINT_URGENT, HINT_POLITE = 1, 2


def _compile(env=None, queue=False):
    from ..compiler.nvptx import CudaModule, compile_ptx
    from ..compiler.weave import weave
    src = open(os.path.join(HERE, "hetero_decode.ll")).read()
    if queue:
        src = src.replace("@__sched_timer = ", "@__sched_queue = addrspace(1) externally_initialized "
                                               "global ptr null, align 8\n@__sched_timer = ")
    if env is not None:
        src, _ = weave(src, env)
    return CudaModule(compile_ptx(src))


class Plane:
    """Device control tables in the ABI layout for one woven module."""

    def __init__(self, n=1024):
        self.n = n
        self.order = torch.arange(n, dtype=torch.int32, device="cuda")
        self.host = bytearray(abi.ctrl_bytes(n))
        self.ctrl = torch.zeros(abi.ctrl_bytes(n), dtype=torch.uint8, device="cuda")
        self.timer = torch.zeros(n, dtype=torch.int64, device="cuda")
        self.queue = torch.zeros(4, dtype=torch.int32, device="cuda")

    def u32(self, off, v):
        self.host[off:off + 4] = int(v).to_bytes(4, "little")

    def hint(self, i, h):
        self.host[abi.CTRL_ROWS_OFF + abi.ROW_SIZE * i + 6] = h

    def push(self):
        self.ctrl.copy_(torch.frombuffer(bytearray(self.host), dtype=torch.uint8))

    def arm(self, mod, queue=False):
        mod.set_global_ptr("__sched_task_order", self.order.data_ptr())
        mod.set_global_ptr("__sched_ctrl", self.ctrl.data_ptr())
        mod.set_global_ptr("__sched_timer", self.timer.data_ptr())
        if queue:
            mod.set_global_ptr("__sched_queue", self.queue.data_ptr())

    def set_order(self, tasks, n):
        o = torch.arange(self.n, dtype=torch.int32)
        o[:len(tasks)] = torch.as_tensor(tasks, dtype=torch.int32)
        self.order.copy_(o.cuda())
        self.u32(abi.CTRL_ORDER_SIZE_OFF, n)


def inputs(nseq=64, longb=32, shortb=4, seed=777):
    g = torch.Generator().manual_seed(seed)
    npages = nseq * longb
    kv = (torch.rand(npages * PT * D + 8192, generator=g) - 0.5).cuda()
    w = (torch.rand(PT, generator=g) - 0.5).cuda()
    is_long = np.array([t % 8 == 0 for t in range(nseq)])
    nbl = torch.tensor(np.where(is_long, longb, shortb), dtype=torch.int32).cuda()
    bt = torch.tensor([[(t * longb + b * 17 + 5) % npages for b in range(longb)] for t in range(nseq)],
                      dtype=torch.int32).cuda()
    return kv, bt, nbl, w, is_long


def run(iters=100, nseq=64, workers=16, longb=32, shortb=4, emit=print) -> dict:
    kv, bt, nbl, w, is_long = inputs(nseq, longb, shortb)
    out = torch.zeros(nseq * D, device="cuda")

    def launch(mod, grid):
        mod.launch("hetero_decode", (grid,), (D,), [kv, bt, nbl, w, out, longb])

    def timed(mod, grid, reset=None):
        if reset:
            reset()
        launch(mod, grid)
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(iters):
            if reset:
                reset()
            launch(mod, grid)
        e.record()
        e.synchronize()
        return 1e3 * s.elapsed_time(e) / iters

    def result(mod, grid, reset=None):
        out.zero_()
        if reset:
            reset()
        launch(mod, grid)
        torch.cuda.synchronize()
        return out.clone()

    stock = _compile()
    golden = result(stock, nseq)
    res = {"static_us": timed(stock, nseq)}

    wq = _compile({"SCHED_WORKQUEUE": "1"}, queue=True)
    p = Plane()
    p.u32(abi.CTRL_NUM_TASKS_OFF, nseq)
    p.push()
    p.arm(wq, queue=True)

    def prime():  # the ticket starts at the worker count (the first W tasks are the workers' own)
        p.queue[0] = workers
        p.queue[1] = 0
    exact = {}

    def arm_run(name, order=None):
        if order is not None:
            p.set_order(order, nseq)
        p.push()
        exact[name] = bool(torch.equal(result(wq, workers, prime), golden))
        res[f"{name}_us"] = timed(wq, workers, prime)

    arm_run("identity", list(range(nseq)))
    arm_run("segregated", [t for t in range(nseq) if not is_long[t]] + [t for t in range(nseq) if is_long[t]])
    # closed loop: one profiling step with the woven timer, then LPT on the measured cycles
    p.set_order(list(range(nseq)), nseq)
    p.push()
    p.timer.zero_()
    result(wq, workers, prime)
    cyc = p.timer[:nseq].cpu().numpy()
    lpt = [int(t) for t in np.argsort(-cyc, kind="stable")]
    res["timer_ranks_longs_first"] = bool(all(is_long[t] for t in lpt[:int(is_long.sum())]))
    arm_run("lpt", lpt)
    for t in range(nseq):
        p.hint(t, HINT_POLITE if is_long[t] else HINT_URGENT)
    arm_run("lpt_hints")
    for t in range(nseq):
        p.hint(t, 0)
    p.push()

    clc = _compile({"SCHED_WORKQUEUE": "1", "SCHED_CLC": "1"})
    pc = Plane()
    pc.u32(abi.CTRL_NUM_TASKS_OFF, nseq)
    pc.set_order(lpt, nseq)
    pc.push()
    pc.arm(clc)
    exact["clc"] = bool(torch.equal(result(clc, nseq), golden))
    res["clc_us"] = timed(clc, nseq)

    res = {k: (round(v, 2) if isinstance(v, float) else v) for k, v in res.items()}
    rec = {"case": "hetero_batch", "tasks": nseq, "workers": workers, "long_blocks": longb, "short_blocks": shortb,
           **res, "bit_exact": exact,
           "reference_a6000_us": {"identity": 405, "lpt": 272, "lpt_hints": 265}}
    emit(json.dumps(rec))
    return rec


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--iters", type=int, default=100)
    ap.add_argument("--workers", type=int, default=16)
    args = ap.parse_args(argv)
    run(args.iters, workers=args.workers)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
