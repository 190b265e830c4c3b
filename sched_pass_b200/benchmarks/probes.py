#!/usr/bin/env python
"""Hardware probes behind the levers (csrc/kernels/microbench.cu).

* ``stream``: one pass over a 4 GiB buffer (32x L2) under each L2 cache
  policy; GB/s and fraction of the measured HBM copy bandwidth. The policy
  lever is kept dormant on decode when no hint moves this number.
* ``tasks``: makespan of a task grid under static grid-stride (R persistent
  CTAs), a ticket queue (R CTAs) and cluster launch control (one CTA per
  task), on uniform, bimodal (straggler) and memory-bound task mixes; every
  run checks that each task executed exactly once.
* ``reuse``: a reused set R (16 MiB .. 256 MiB) read 1:1 with a 2 GiB stream
  S, plain loads vs R pinned (evict_last) and S streamed (evict_first): does
  cache management pay once a stream floods a reused set?
* ``budget``: R = 192 MiB (> L2), the pinned fraction f of R swept from
  0.125 to 1: is L2 residency a continuous per-request budget?
* ``pdl``: producer -> consumer pairs with and without programmatic stream
  serialization, consumer prologue 0 / 256 FMAs; us per pair.
* ``clc``: cluster launch control as the CTAs see it (one CTA per task):
  cycles a CTA waits for a successful claim's answer (late bound: the claim
  issued after the body), exactly one failed claim per worker and exactly-once
  coverage, the number of workers against the resident prefix R, and the
  makespan of static / CLC late-bound / CLC claim-ahead on uniform,
  long-suffix, long-prefix and interleaved layouts (8192 tasks of 1024
  cycles, a quarter 32x longer).

    python -m sched_pass_b200.benchmarks.probes [--only stream|tasks|reuse|budget|pdl]
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


MIX_MODES = ["lru", "pin_R_stream_S", "pin_R_rest_first"]


def _mix(R, S, mode, frac, sink, grid):
    return _time(lambda: ext().probe_mix(R, S, mode, frac, sink, grid))


def reuse(s_gib: float = 2.0):
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    S = torch.randint(0, 1 << 30, (int(s_gib * (1 << 28)),), dtype=torch.int32, device="cuda")
    sink = torch.zeros(1 << 16, dtype=torch.int32, device="cuda")
    s_bytes = S.numel() * 4
    out = []
    for r_mib in (16, 32, 64, 96, 128, 192, 256):
        R = torch.randint(0, 1 << 30, (r_mib << 18,), dtype=torch.int32, device="cuda")
        for mode in (0, 1):
            ms = _mix(R, S, mode, 1.0, sink, sms * 4)
            # every iteration reads one R vector and one S vector: 2 x |S| bytes requested;
            # if R stays in L2 only |S| comes from DRAM
            rec = {"probe": "reuse", "R_MiB": r_mib, "S_GiB": s_gib, "mode": MIX_MODES[mode], "ms": round(ms, 3),
                   "requested_GBps": round(2 * s_bytes / ms / 1e6, 1),
                   "dram_GBps_if_R_hits": round(s_bytes / ms / 1e6, 1)}
            print(json.dumps(rec), flush=True)
            out.append(rec)
        del R
    return out


def budget(r_mib: int = 192, s_gib: float = 2.0):
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    S = torch.randint(0, 1 << 30, (int(s_gib * (1 << 28)),), dtype=torch.int32, device="cuda")
    R = torch.randint(0, 1 << 30, (r_mib << 18,), dtype=torch.int32, device="cuda")
    sink = torch.zeros(1 << 16, dtype=torch.int32, device="cuda")
    out = []
    base = _mix(R, S, 0, 1.0, sink, sms * 4)
    print(json.dumps({"probe": "budget", "R_MiB": r_mib, "mode": "lru", "ms": round(base, 3)}), flush=True)
    for mode in (1, 2):
        for f in (0.125, 0.25, 0.375, 0.5, 0.625, 0.75, 1.0):
            ms = _mix(R, S, mode, f, sink, sms * 4)
            rec = {"probe": "budget", "R_MiB": r_mib, "mode": MIX_MODES[mode], "pin_fraction": f,
                   "pinned_MiB": round(f * r_mib, 1), "ms": round(ms, 3), "vs_lru": round(ms / base, 3)}
            print(json.dumps(rec), flush=True)
            out.append(rec)
    return out


def pdl(n: int = 148 * 256 * 4, pairs: int = 200):
    buf = torch.zeros(n, device="cuda")
    out_ = torch.zeros(n, device="cuda")
    table = torch.rand(256, device="cuda")
    res = []
    for work in (64, 1024):
        for prologue in (0, 256):
            row = {"probe": "pdl", "threads": n, "producer_fmas": work, "consumer_prologue_fmas": prologue}
            for on in (False, True):
                ms = _time(lambda: ext().probe_pdl_pairs(buf, out_, table, work, prologue, on, pairs))
                row["us_per_pair_" + ("pdl" if on else "plain")] = round(ms * 1e3 / pairs, 2)
            row["saved_us_per_pair"] = round(row["us_per_pair_plain"] - row["us_per_pair_pdl"], 2)
            print(json.dumps(row), flush=True)
            res.append(row)
    return res


CLC_MODES = ["static", "clc_late", "clc_ahead"]


def clc_layout(n: int, base: int, name: str, long_frac: float = 0.25, factor: int = 32) -> np.ndarray:
    """Per-task body cycles: uniform, or a quarter of the tasks ``factor``x
    longer at the end (long-suffix), the start (long-prefix) or every
    fourth task (interleaved)."""
    w = np.full(n, base, dtype=np.int64)
    k = int(n * long_frac)
    if name == "long_suffix":
        w[n - k:] *= factor
    elif name == "long_prefix":
        w[:k] *= factor
    elif name == "interleaved":
        w[::int(round(1 / long_frac))] *= factor
    elif name != "uniform":
        raise ValueError(name)
    return w.astype(np.int32)


def run_clc(work: np.ndarray, mode: int, R: int, max_rec: int = 16):
    """One probe launch; returns (ms, hits, rec [grid, max_rec] int64, n_rec, smid)."""
    n = work.size
    grid = R if mode == 0 else n
    w = torch.from_numpy(work).cuda()
    hits = torch.zeros(n, dtype=torch.int32, device="cuda")
    rec = torch.zeros(grid, max_rec, dtype=torch.int64, device="cuda")
    n_rec = torch.zeros(grid, dtype=torch.int32, device="cuda")
    smid = torch.full((grid,), -1, dtype=torch.int32, device="cuda")
    st = ops.status_buffer()

    def go():
        hits.zero_()
        n_rec.zero_()
        ext().probe_clc(w, mode, grid, hits, rec, n_rec, smid, st)
    ms = _time(go)
    go()
    torch.cuda.synchronize()
    ops.check_status()
    return ms, hits.cpu().numpy(), rec.cpu().numpy(), n_rec.cpu().numpy(), smid.cpu().numpy()


def clc_claims(rec: np.ndarray, n_rec: np.ndarray):
    """Per worker (a CTA that ran): its claims as (waited cycles, value)."""
    out = {}
    for c in np.flatnonzero(n_rec > 0):
        k = min(int(n_rec[c]), rec.shape[1])
        r = rec[c, :k].astype(np.uint64)
        out[int(c)] = [(int(x >> np.uint64(32)), int(x & np.uint64(0xFFFFFFFF))) for x in r]
    return out


def clc(n: int = 8192, base: int = 1024):
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    occ = int(ext().probe_tasks_occupancy())
    R = occ * sms
    FAIL = 0xFFFFFFFF
    # claim latency and the terminal-failure rule on uniform work
    _, hits, rec, n_rec, smid = run_clc(clc_layout(n, base, "uniform"), 1, R)
    claims = clc_claims(rec, n_rec)
    ok_wait = sorted(w for cl in claims.values() for w, x in cl if x != FAIL)
    terminal = [sum(1 for _, x in cl if x == FAIL) for cl in claims.values()]
    last_is_fail = all(cl and cl[-1][1] == FAIL for cl in claims.values())
    claimed = sorted(x for cl in claims.values() for _, x in cl if x != FAIL)
    pct = lambda v, q: int(v[min(len(v) - 1, int(q * len(v)))]) if v else None  # noqa: E731
    rec_out = {"probe": "clc_claims", "tasks": n, "R": R, "workers": len(claims),
               "successes": len(claimed), "expected_successes": max(0, n - len(claims)),
               "failures_per_worker_min": min(terminal), "failures_per_worker_max": max(terminal),
               "failure_is_last_claim": last_is_fail,
               "every_task_once": bool((hits == 1).all()), "claims_unique": len(set(claimed)) == len(claimed),
               "claim_wait_cycles_p50": pct(ok_wait, 0.5), "claim_wait_cycles_p90": pct(ok_wait, 0.9),
               "claim_wait_cycles_p99": pct(ok_wait, 0.99),
               "distinct_sms": int(len(set(int(s) for s in smid[n_rec > 0])))}
    print(json.dumps(rec_out), flush=True)
    # placement: static vs late-bound vs claim-ahead
    for layout in ("uniform", "long_suffix", "long_prefix", "interleaved"):
        work = clc_layout(n, base, layout)
        row = {"probe": "clc_placement", "layout": layout, "tasks": n, "body_cycles": base}
        for mode, name in enumerate(CLC_MODES):
            ms, hits, rec, n_rec, _ = run_clc(work, mode, R)
            row[name + "_us"] = round(ms * 1e3, 2)
            row[name + "_exactly_once"] = bool((hits == 1).all())
            if mode == 2:
                cl = clc_claims(rec, n_rec)
                waits = sorted(w for c in cl.values() for w, x in c if x != FAIL)
                row["clc_ahead_collect_wait_p50"] = pct(waits, 0.5)
            if mode == 1:
                cl = clc_claims(rec, n_rec)
                waits = sorted(w for c in cl.values() for w, x in c if x != FAIL)
                row["clc_late_claim_wait_p50"] = pct(waits, 0.5)
        st = row["static_us"]
        row["late_vs_static"] = round(row["clc_late_us"] / st - 1, 4)
        row["ahead_vs_static"] = round(row["clc_ahead_us"] / st - 1, 4)
        print(json.dumps(row), flush=True)


def run_clc_shape(work: np.ndarray, gx: int, gy: int = 1, gz: int = 1, stride: int = 1, cx: int = 1,
                  graph_replays: int = 0):
    """One launch (or ``graph_replays`` replays of a CUDA graph holding the
    counter reset and the launch) of the CLC shape probe; returns the
    contract figures of the last run."""
    n = gx * gy * gz
    w = torch.from_numpy(work[:n]).cuda()
    counters = torch.zeros(4 * n + 1, dtype=torch.int32, device="cuda")
    st = ops.status_buffer()

    def go():
        counters.zero_()
        ext().probe_clc_shape(w, gx, gy, gz, stride, cx, counters, st)
    runs = []
    if graph_replays:
        go()  # warm-up outside the capture
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            go()
        for _ in range(graph_replays):
            g.replay()
            torch.cuda.synchronize()
            runs.append(counters.cpu().numpy().astype(np.int64))
        del g
    else:
        go()
        torch.cuda.synchronize()
        runs.append(counters.cpu().numpy().astype(np.int64))
    ops.check_status()
    out = []
    for c in runs:
        hits, claimed, launched, fails = c[:n], c[n:2 * n], c[2 * n:3 * n], c[3 * n:4 * n]
        cl = np.flatnonzero(claimed > 0)
        workers = np.flatnonzero((launched > 0) & (np.arange(n) % (stride * cx) == 0))
        holes = int(cl[-1] - cl[0] + 1 - cl.size) if cl.size else 0
        out.append({
            "tasks": n, "exactly_once": bool((hits == 1).all()), "duplicate_claims": int((claimed > 1).sum()),
            "launched": int((launched > 0).sum()), "claimed": int(cl.size),
            "claimed_min": int(cl[0]) if cl.size else None, "claimed_max": int(cl[-1]) if cl.size else None,
            "claim_holes": holes, "claim_bases_aligned": bool((cl[cl % cx == 0].size * cx == cl.size)) if cx > 1 else True,
            "claiming_workers": int(workers.size),
            "failures_per_worker": sorted(set(int(f) for f in fails[workers])) if workers.size else [],
            "w_nonzero": int(c[4 * n])})
    return out


def clc_shapes(base: int = 1024):
    """The CLC contract under 2-D / 3-D grids, partial participation,
    clustered launches and CUDA-graph replay (one JSON line per case)."""
    R = int(ext().probe_clc_shape_capacity(1))
    cases = [("1d", dict(gx=8192)), ("2d_64x128", dict(gx=64, gy=128)), ("3d_17x19x29", dict(gx=17, gy=19, gz=29)),
             ("stride2", dict(gx=8192, stride=2)), ("stride4", dict(gx=8192, stride=4)),
             ("cluster2", dict(gx=8192, cx=2)), ("cluster4", dict(gx=8192, cx=4)),
             ("graph_replay", dict(gx=8192, graph_replays=5))]
    rows = []
    for name, kw in cases:
        n = kw["gx"] * kw.get("gy", 1) * kw.get("gz", 1)
        work = np.full(n, base, dtype=np.int32)
        res = run_clc_shape(work, **kw)
        cx = kw.get("cx", 1)
        pred = int(ext().probe_clc_shape_capacity(cx)) if cx > 1 else R
        row = {"probe": "clc_shape", "case": name, "predicted_R": pred, **res[-1]}
        if len(res) > 1:
            row["replays"] = len(res)
            row["replays_identical_contract"] = all(
                r["exactly_once"] and r["claimed_min"] == res[0]["claimed_min"] and r["claim_holes"] == 0 for r in res)
        print(json.dumps(row), flush=True)
        rows.append(row)
    return rows


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--only", choices=["stream", "tasks", "reuse", "budget", "pdl", "clc", "clc_shapes"])
    a = ap.parse_args(argv)
    if a.only in (None, "stream"):
        stream()
    if a.only in (None, "tasks"):
        tasks()
    if a.only in (None, "reuse"):
        reuse()
    if a.only in (None, "budget"):
        budget()
    if a.only in (None, "pdl"):
        pdl()
    if a.only in (None, "clc"):
        clc()
    if a.only in (None, "clc_shapes"):
        clc_shapes()


if __name__ == "__main__":
    main()
