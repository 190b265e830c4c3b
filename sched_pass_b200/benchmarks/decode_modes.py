"""Single-GPU paged-decode fixture in every lever mode (the 1xB200 config).

Shape: bf16, 256 requests, 32 query heads, 8 KV heads, head_dim 128, page
size 16, pages shuffled randomly, context lengths lognormal (median 1024,
sigma 1.0, clipped to [64, 32768]), Q/K/V ~ N(0,1), urgency q ~ U[0,1].

Modes (one task = one (request, KV head); no KV splitting, so long requests
are stragglers and scheduling matters):
  stock    unwoven kernel, identity order
  woven    levers compiled in, tables neutral (bit-exact with stock)
  unarmed  levers compiled in, no tables bound (what the woven code costs
           without any table read)
  pi       LPT order (grouped, block 16)
  policy   urgency rows + hints (urgent tasks prefetch / evict_last)
  timer    per-task timer on
  shed     tau = 0.5 * length for every request
  ticket   persistent workers (R = occupancy x SMs), atomic ticket, LPT order
  clc      grid = tasks, cluster-launch-control stealing, region order
  split    KV split 4 ways + merge (for reference)
  flashinfer  the installed FlashInfer library's BatchDecodeWithPagedKVCache
           (the kernel the reference weaves into SGLang: jc-su/sched-pass
           SGLANG.md, test/py/test_flashinfer_arm.py) on the same pages, HND
           layout; run as a library only, its output checked against stock
Each mode: median device time over iterations with an L2 flush between them,
achieved KV bandwidth vs the measured HBM peak, and bit-exactness vs stock
for the permutation-only modes. ``--trace`` adds each mode's per-CTA phase
trace of one launch (after an L2 flush).
"""
from __future__ import annotations

import argparse
import json
import math

import numpy as np
import torch

from .. import ops
from ..engine import native
from ..runtime.sched_rt import SchedPlane
from .common import L2Flusher, measured_peaks, time_fn


def build(B=256, Hq=32, Hkv=8, seed=0, median=1024, sigma=1.0, lo=64, hi=32768):
    rng = np.random.default_rng(seed)
    lens = np.clip(np.round(median * np.exp(sigma * rng.standard_normal(B))), lo, hi).astype(np.int32)
    pages_per = (lens + 15) // 16
    total = int(pages_per.sum())
    perm = rng.permutation(total).astype(np.int32)
    maxp = int(pages_per.max())
    bt = np.zeros((B, maxp), dtype=np.int32)
    k = 0
    for b in range(B):
        bt[b, :pages_per[b]] = perm[k:k + pages_per[b]]
        k += pages_per[b]
    g = torch.Generator(device="cuda").manual_seed(seed)
    kc = torch.randn(total, Hkv, 16, 128, device="cuda", generator=g).to(torch.bfloat16)
    vc = torch.randn(total, Hkv, 16, 128, device="cuda", generator=g).to(torch.bfloat16)
    q = torch.randn(B, Hq, 128, device="cuda", generator=g).to(torch.bfloat16)
    urg = rng.random(B).astype(np.float32)
    return lens, torch.from_numpy(bt).cuda(), kc, vc, q, urg


def flashinfer_decode(lens, bt, kc, vc, q, Hq, Hkv, scale):
    """A closure running FlashInfer's paged decode over this fixture's pages
    (indptr / indices / last-page lengths from the block table), or None if
    the library cannot plan it here."""
    try:
        import flashinfer
    except ImportError:
        return None
    pages = (lens + 15) // 16
    indptr = np.concatenate([[0], np.cumsum(pages)]).astype(np.int32)
    btn = bt.cpu().numpy()
    indices = np.concatenate([btn[b, :pages[b]] for b in range(len(lens))]).astype(np.int32)
    last = (lens - (pages - 1) * 16).astype(np.int32)
    ws = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    w = flashinfer.BatchDecodeWithPagedKVCacheWrapper(ws, kv_layout="HND")
    try:
        w.plan(torch.from_numpy(indptr).cuda(), torch.from_numpy(indices).cuda(), torch.from_numpy(last).cuda(),
               Hq, Hkv, 128, 16, q_data_type=torch.bfloat16, kv_data_type=torch.bfloat16, sm_scale=scale)
    except Exception as e:  # noqa: BLE001 - report, do not fail the other modes
        print(json.dumps({"mode": "flashinfer", "plan_error": repr(e)[:300]}))
        return None
    fo = torch.empty_like(q)

    def run():
        return w.run(q, (kc, vc), out=fo)
    return run


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--requests", type=int, default=256)
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--modes", default="stock,woven,pi,policy,timer,shed,ticket,clc,split,flashinfer")
    ap.add_argument("--trace", action="store_true", help="per-CTA phase trace of one launch per mode")
    args = ap.parse_args()
    Hq, Hkv = 32, 8
    lens, bt, kc, vc, q, urg = build(args.requests, Hq, Hkv)
    B = len(lens)
    items, _, _ = native.plan_decode(lens, 1)
    items_t = torch.from_numpy(items).cuda()
    n_items = items.shape[0]
    n_tasks = n_items * Hkv
    cost = native.task_costs(items, n_items, Hkv)
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    occ = ops.kernels.ext().attn_decode_occupancy(Hq // Hkv)
    R = occ * sms
    plane = SchedPlane(max_tasks=max(n_tasks, 64), device="cuda", mode="device")
    out = torch.empty_like(q)
    scale = 1.0 / math.sqrt(128)
    flush = L2Flusher("cuda")
    peaks = measured_peaks()
    kv_bytes = float(lens.astype(np.int64).sum()) * Hkv * 128 * 2 * 2

    def reset_plane():
        plane.reset_order()
        plane.set_order_size(0)
        plane.set_num_tasks(0)
        plane.set_timer_enabled(False)
        plane.set_rows(n=n_tasks)
        plane.push()

    def run(woven, acquire=0, grid=0, slots=True):
        ops.attention_decode(q, out, kc, vc, bt, items_t, n_items, scale,
                             slots=plane.slots() if (woven and slots) else None, woven=woven,
                             acquire=acquire, grid=grid)

    from ..utils.clocks import ClockSampler
    sampler = ClockSampler(gpu_index=torch.cuda.current_device()).start()
    results = {}
    stock_out = None
    for mode in args.modes.split(","):
        reset_plane()
        kv = kv_bytes
        if mode == "stock":
            fn = lambda: run(False)
        elif mode == "woven":
            fn = lambda: run(True)
        elif mode == "unarmed":
            fn = lambda: run(True, slots=False)
        elif mode == "pi":
            plane.install_order(torch.from_numpy(native.grouped_lpt(cost, 16)), n_tasks)
            plane.push()
            fn = lambda: run(True)
        elif mode == "policy":
            hint = np.zeros(n_tasks, dtype=np.int64)
            plane.set_rows(q=np.repeat(urg, Hkv), hint=hint, n=n_tasks)
            plane.set_lambda(bw=0.25)
            plane.push()
            fn = lambda: run(True)
        elif mode == "timer":
            plane.set_timer_enabled(True)
            plane.push()
            fn = lambda: run(True)
        elif mode == "shed":
            tau = np.repeat(np.maximum(1, lens // 2), Hkv)
            plane.set_rows(tau=tau, n=n_tasks)
            plane.push()
            kv = float(np.maximum(1, lens // 2).astype(np.int64).sum()) * Hkv * 128 * 4
            fn = lambda: run(True)
        elif mode == "ticket":
            plane.install_order(torch.from_numpy(native.grouped_lpt(cost, 1)), n_tasks)
            plane.set_num_tasks(n_tasks)
            plane.push()
            fn = lambda: run(True, acquire=1, grid=R)
        elif mode == "clc":
            plane.install_order(torch.from_numpy(native.region_order(cost, R, 16)), n_tasks)
            plane.set_num_tasks(n_tasks)
            plane.push()
            fn = lambda: run(True, acquire=2)
        elif mode == "split":
            it4, mreq, mbeg = native.plan_decode(lens, 4)
            it4_t = torch.from_numpy(it4).cuda()
            po = torch.empty(B * 4, Hq, 128, dtype=torch.float32, device="cuda")
            pl = torch.empty(B * 4, Hq, dtype=torch.float32, device="cuda")
            mr = torch.from_numpy(mreq).cuda()
            mb = torch.from_numpy(mbeg).cuda()

            def fn():
                ops.attention_decode(q, out, kc, vc, bt, it4_t, it4.shape[0], scale, part_o=po,
                                     part_lse=pl, woven=False)
                ops.attention_merge(po, pl, mr, mb, B, out)
        elif mode == "flashinfer":
            fn = flashinfer_decode(lens, bt, kc, vc, q, Hq, Hkv, scale)
            if fn is None:
                print(json.dumps({"mode": mode, "unavailable": "flashinfer decode could not be planned"}))
                continue
        else:
            raise ValueError(mode)
        ms = time_fn(fn, args.iters, flush=flush)
        fn()
        torch.cuda.synchronize()
        rec = {"mode": mode, "us": round(ms * 1e3, 1), "kv_GBps": round(kv / ms / 1e6, 1),
               "frac_hbm_of_measured": round(kv / ms / 1e6 / peaks["hbm_gbs"], 3)}
        if mode == "flashinfer" and stock_out is not None:
            fo = fn()
            torch.cuda.synchronize()
            rec["rel_err_vs_stock"] = round(float((fo.float() - stock_out.float()).norm() /
                                                  stock_out.float().norm()), 5)
        if mode == "stock":
            stock_out = out.clone()
        elif mode in ("woven", "unarmed", "pi", "timer", "ticket", "clc", "policy") and stock_out is not None:
            rec["bit_exact_vs_stock"] = bool(torch.equal(out, stock_out))
        if args.trace and mode not in ("split", "flashinfer"):
            from .kernel_cases import decode_trace
            flush()
            rec["phases"] = decode_trace(fn, R if mode == "ticket" else n_tasks)
        if mode == "timer":
            cyc = plane.read_timer()[:n_tasks].double()
            rec["timer_rows_filled"] = int((cyc > 0).sum())
        results[mode] = rec
        print(json.dumps(rec), flush=True)
    ops.check_status()
    print(json.dumps({"clocks": sampler.stop()}))
    print(json.dumps({"requests": B, "tasks": n_tasks, "R": R, "occupancy": occ,
                      "kv_GB": round(kv_bytes / 1e9, 3), "len_p50": int(np.median(lens)),
                      "len_max": int(lens.max())}))


if __name__ == "__main__":
    main()
