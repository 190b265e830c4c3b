#!/usr/bin/env python
"""Hardware probes behind the levers (csrc/kernels/microbench.cu).

* ``stream``: one pass over a 4 GiB buffer (32x L2) under each L2 cache
  policy; GB/s and fraction of the measured HBM copy bandwidth. The policy
  lever is kept dormant on decode when no hint moves this number.
* ``tasks``: makespan of a task grid under static grid-stride (R persistent
  CTAs), a ticket queue (R CTAs) and cluster launch control (one CTA per
  task), on uniform, bimodal (straggler) and memory-bound task mixes; every
  run checks that each task executed exactly once.

    python -m sched_pass_b200.benchmarks.probes [--only stream|tasks]
"""
from __future__ import annotations

import argparse
import json

import numpy as np
import torch

from .._ext import ext
from .. import ops
from .common import measured_peaks

POLICIES = ["none", "evict_first", "evict_last", "evict_normal", "evict_unchanged"]
MODES = ["static", "ticket", "clc"]


def _time(fn, iters=5):
    fn()
    torch.cuda.synchronize()
    ts = []
    for _ in range(iters):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        fn()
        b.record()
        b.synchronize()
        ts.append(a.elapsed_time(b))
    return float(np.median(ts))


def stream(gib: float = 4.0):
    n = int(gib * (1 << 30))
    src = torch.randint(0, 1 << 30, (n // 4,), dtype=torch.int32, device="cuda")
    sink = torch.zeros(1 << 16, dtype=torch.int32, device="cuda")
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    hbm = measured_peaks().get("hbm_gbs", 6543.0)
    out = []
    for pol, name in enumerate(POLICIES):
        ms = _time(lambda: ext().probe_stream(src, pol, sink, sms * 4))
        gbs = n / ms / 1e6
        # the measured peak counts read + write bytes of a copy; a read-only
        # stream is compared against it as is
        rec = {"probe": "stream", "policy": name, "bytes": n, "ms": round(ms, 3), "GBps": round(gbs, 1),
               "frac_of_measured_copy": round(gbs / hbm, 3)}
        print(json.dumps(rec), flush=True)
        out.append(rec)
    return out


def run_tasks(cost: np.ndarray, mode: int, memory: bool, R: int, data):
    n = cost.size
    c = torch.from_numpy(cost.astype(np.int32)).cuda()
    hits = torch.zeros(n, dtype=torch.int32, device="cuda")
    per_cta = torch.zeros(max(n, R), dtype=torch.int32, device="cuda")
    ticket = torch.zeros(1, dtype=torch.int32, device="cuda")
    sink = torch.zeros(4, dtype=torch.int32, device="cuda")
    st = ops.status_buffer()

    def go():
        hits.zero_()
        per_cta.zero_()
        ticket.zero_()
        ext().probe_tasks(c, mode, R, int(memory), data, hits, per_cta, ticket, sink, st)

    ms = _time(go, 3)
    ops.check_status()
    h = hits.cpu().numpy()
    pc = per_cta.cpu().numpy()
    used = pc[pc > 0]
    return ms, bool((h == 1).all()), float(used.max() / used.mean()) if used.size else 0.0


def tasks():
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    R = ext().probe_tasks_occupancy() * sms
    rng = np.random.default_rng(0)
    data = torch.zeros(1 << 28, dtype=torch.int32, device="cuda")  # 1 GiB for memory-bound tasks
    mixes = {}
    n = 4 * R
    mixes["uniform_20us"] = (np.full(n, 20000), False)
    bim = np.full(n, 20000)
    bim[rng.choice(n, n // 10, replace=False)] = 200000
    mixes["bimodal_10pct_10x"] = (bim, False)
    mixes["bimodal_at_R"] = (np.where(np.arange(R) < R // 16, 400000, 20000), False)
    mixes["memory_1MiB"] = (np.full(n, 1 << 20), True)
    out = []
    for name, (cost, mem) in mixes.items():
        ideal = cost.sum() / (R if not mem else 1) / 1e6 if not mem else None
        for m, mname in enumerate(MODES):
            ms, exact, imb = run_tasks(cost, m, mem, R, data)
            rec = {"probe": "tasks", "mix": name, "mode": mname, "tasks": int(cost.size), "R": R,
                   "makespan_ms": round(ms, 4), "exactly_once": exact, "per_cta_max_over_mean": round(imb, 3)}
            if ideal:
                rec["lower_bound_ms"] = round(max(ideal, cost.max() / 1e6), 4)
            print(json.dumps(rec), flush=True)
            out.append(rec)
    return out


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--only", choices=["stream", "tasks"])
    a = ap.parse_args(argv)
    if a.only in (None, "stream"):
        stream()
    if a.only in (None, "tasks"):
        tasks()


if __name__ == "__main__":
    main()
