"""Small standalone cases of single kernels, for device timing and for
``ncu`` captures of one launch (inputs above L2 where the kernel streams,
a few hundred MB on the device at most).

  --case sp_norm   sequence-parallel reduce + residual + RMSNorm + all-gather
                   (``sp_reduce_norm_kernel``) for W ranks emulated on one
                   GPU: every rank's reduce-scatter GEMM runs first, then the
                   owners' norms, so no launch waits on a later one
  --case prefill   causal paged prefill attention of one 1536-token prompt
                   (Llama-3-8B heads: 32 query / 8 KV, head_dim 128)
  --case sample    embedding gather (T tokens) and greedy argmax over the
                   128256-entry vocabulary
  --case decode    the serving engine's decode attention launch for a small
                   batch (``--batch`` requests of ``--context`` tokens, 4
                   query heads per KV head, ``--kv-heads`` KV heads, pages scattered over a
                   pool larger than L2): KV split the way the engine splits it
                   (tasks up to one per SM), in-kernel merge, levers woven
                   with neutral tables, cluster launch control grid

Prints one JSON line per case with the median device time (CUDA events,
after warm-up) and the algorithmic bytes / FLOPs per launch.
"""
from __future__ import annotations

import argparse
import json
import math

import torch

from .. import ops
from .._ext import ext
from .common import measured_peaks


def events_ms(fn, reps):
    fn()
    torch.cuda.synchronize()
    ts = []
    for _ in range(reps):
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        fn()
        e.record()
        e.synchronize()
        ts.append(s.elapsed_time(e))
    return sorted(ts)[len(ts) // 2]


def case_sp_norm(args, peaks):
    W, T, H, K = args.world, args.tokens, 4096, 2048
    M = (T + 3) // 4 * 4
    dev = "cuda"
    z = lambda *s, dt=torch.bfloat16: torch.zeros(*s, dtype=dt, device=dev)  # noqa: E731
    slab = [z(W, M, H) for _ in range(W)]
    rflags = [z(W * (H // 128) * M, dt=torch.int32) for _ in range(W)]
    gather = [[z(M, H) for _ in range(W)] for _ in range(2)]
    ready = [[z(M, dt=torch.int32) for _ in range(W)] for _ in range(2)]
    xs = [torch.randn(T, K, device=dev).to(torch.bfloat16) for _ in range(W)]
    ws = [(torch.randn(H, K, device=dev) / math.sqrt(K * W)).to(torch.bfloat16) for _ in range(W)]
    res = [torch.randn(T, H, device=dev).to(torch.bfloat16) for _ in range(W)]
    lnw = torch.ones(H, dtype=torch.bfloat16, device=dev)
    st = ops.status_buffer()
    ptrs = lambda lst: [t.data_ptr() for t in lst]  # noqa: E731
    k = [0]

    def push():
        for r in range(W):
            w_ = ops.kernels._ws_for(xs[r], H, K, 0, None)
            ext().gemm_reduce_scatter(xs[r], ws[r], r, W, ptrs(slab), ptrs(rflags), 0, w_.ws, w_.counters, st)

    def norms():
        g = k[0]
        for r in range(W):
            ext().sp_reduce_norm(slab[r].data_ptr(), rflags[r].data_ptr(), res[r], lnw, None, ptrs(gather[g]),
                                 ptrs(ready[g]), ready[g ^ 1][r].data_ptr(), M, T, r, W, 1e-5, st)
        k[0] ^= 1

    ts = []
    for _ in range(args.reps):
        push()
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        norms()
        e.record()
        e.synchronize()
        ts.append(s.elapsed_time(e) / W)
    ops.check_status()
    ms = sorted(ts)[len(ts) // 2]
    rows = T / W
    byts = rows * H * 2 * (W + 2 + W)  # partials in, residual in/out, W gathered copies out
    print(json.dumps({"case": "sp_norm", "world": W, "T": T, "H": H, "us_per_rank": round(ms * 1e3, 2),
                      "bytes_per_rank": int(byts), "GBps": round(byts / (ms * 1e-3) / 1e9, 1),
                      "frac_hbm_of_measured": round(byts / (ms * 1e-3) / 1e9 / peaks["hbm_gbs"], 3)}))


def case_prefill(args, peaks):
    T, Hq, Hkv, D, PS = 1536, 32, 8, 128, 16
    pages = T // PS
    dev = "cuda"
    q = torch.randn(T, Hq, D, device=dev).to(torch.bfloat16)
    out = torch.empty_like(q)
    kc = torch.randn(pages, Hkv, PS, D, device=dev).to(torch.bfloat16)
    vc = torch.randn_like(kc)
    bt = torch.randperm(pages, device=dev).to(torch.int32).view(1, pages)
    kvl = torch.tensor([T], dtype=torch.int32, device=dev)
    R = ops.PREFILL_TILE_ROWS
    tiles = torch.tensor([[0, t0, min(R, T - t0), t0] for t0 in range(T - (T - 1) % R - 1, -1, -R)],
                         dtype=torch.int32, device=dev)  # longest first
    fn = lambda: ops.attention_prefill(q, out, kc, vc, bt, kvl, tiles, tiles.shape[0], 1 / math.sqrt(D))  # noqa: E731
    ms = events_ms(fn, args.reps)
    flops = 4 * (T * (T + 1) / 2) * Hq * D  # causal QK^T and PV
    print(json.dumps({"case": "prefill", "T": T, "us": round(ms * 1e3, 2), "TFLOPs": round(flops / (ms * 1e-3) / 1e12, 1),
                      "frac_bf16_of_measured": round(flops / (ms * 1e-3) / 1e12 / peaks["bf16_tflops"], 3)}))


def case_sample(args, peaks):
    V, H = 128256, 4096
    dev = "cuda"
    table = torch.randn(V, H, device=dev).to(torch.bfloat16)
    ids = torch.randint(0, V, (args.tokens,), device=dev, dtype=torch.int32)
    out = torch.empty(args.tokens, H, dtype=torch.bfloat16, device=dev)
    ms_e = events_ms(lambda: ops.embedding(ids, table, out), args.reps)
    logits = torch.randn(128, V, device=dev).to(torch.bfloat16)
    ms_a = events_ms(lambda: ops.argmax(logits), args.reps)
    ops.check_status()
    print(json.dumps({"case": "sample", "embedding_T": args.tokens, "embedding_us": round(ms_e * 1e3, 2),
                      "embedding_GBps": round(2 * args.tokens * H * 2 / (ms_e * 1e-3) / 1e9, 1),
                      "argmax_rows": 128, "argmax_us": round(ms_a * 1e3, 2),
                      "argmax_GBps": round(128 * V * 2 / (ms_a * 1e-3) / 1e9, 1)}))


def case_decode(args, peaks):
    import numpy as np

    from ..engine import native
    from ..runtime.sched_rt import SchedPlane
    # Llama-3-8B's 4 query heads per KV head (a TP rank of 8 GPUs holds 1 KV head)
    B, ctx, Hkv, D = args.batch, args.context, args.kv_heads, 128
    Hq = 4 * Hkv
    dev = "cuda"
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    S = int(min(8, max(1, sms // (B * Hkv))))  # the engine's split rule (Engine.splits_for)
    pool = max(4096, 2 * B * (ctx + 15) // 16)  # pages: K + V pools of ~256 MB, above L2
    kc = torch.randn(pool, Hkv, 16, D, device=dev).to(torch.bfloat16)
    vc = torch.randn_like(kc)
    npg = (ctx + 15) // 16
    bt = torch.randperm(pool, device=dev)[: B * npg].to(torch.int32).view(B, npg)
    lens = np.full(B, ctx, dtype=np.int32)
    items, _, _ = native.plan_decode(lens, S)
    items_t = torch.from_numpy(items).to(dev)
    q = torch.randn(B, Hq, D, device=dev).to(torch.bfloat16)
    out = torch.empty_like(q)
    part_o = torch.zeros(B * S, Hq, D, dtype=torch.float32, device=dev)
    part_lse = torch.zeros(B * S, Hq, dtype=torch.float32, device=dev)
    merge_cnt = torch.zeros(B * Hkv, dtype=torch.int32, device=dev)
    plane = SchedPlane(max_tasks=max(64, items.shape[0] * Hkv), device=dev, mode="device")
    plane.push()
    n_items = items.shape[0]
    fn = lambda: ops.attention_decode(q, out, kc, vc, bt, items_t, n_items, 1 / math.sqrt(D),  # noqa: E731
                                      part_o=part_o if S > 1 else None, part_lse=part_lse if S > 1 else None,
                                      merge_cnt=merge_cnt if S > 1 else None, splits=S, slots=plane.slots(),
                                      woven=True, acquire=2, grid=n_items * Hkv)
    ms = events_ms(fn, args.reps)
    ops.check_status()
    phases = decode_trace(fn, n_items * Hkv) if args.trace else None
    kv = B * ctx * Hkv * D * 2 * 2
    print(json.dumps({"case": "decode", "batch": B, "context": ctx, "kv_heads": Hkv, "splits": S,
                      "tasks": n_items * Hkv, "us": round(ms * 1e3, 2), "kv_MB": round(kv / 1e6, 1),
                      "frac_hbm_of_measured": round(kv / (ms * 1e-3) / 1e9 / peaks["hbm_gbs"], 3),
                      "phases_us": phases}))


DECODE_PHASES = ["setup_and_dep_wait", "task_published", "first_loads_issued", "first_s_tile", "blocks",
                 "output_and_merge", "exit"]


def decode_trace(fn, grid):
    """One launch with the decode kernel's per-CTA %globaltimer trace armed:
    median and max over CTAs of each phase (us), the spread of CTA entries
    and the span from the first entry to the last exit."""
    buf = torch.zeros(grid * 8, dtype=torch.int64, device="cuda")
    torch.cuda.synchronize()
    ext().set_attn_trace(buf.data_ptr())
    try:
        fn()
        torch.cuda.synchronize()
    finally:
        ext().set_attn_trace(0)
    rows = [[int(v) for v in r] for r in buf.view(-1, 8).tolist() if r[0] != 0 and r[7] != 0]
    if not rows:
        return None
    out = {}
    for k, name in enumerate(DECODE_PHASES):
        d = sorted(r[k + 1] - r[k] for r in rows if r[k + 1] and r[k])
        if d:
            out[name] = {"p50": round(d[len(d) // 2] / 1e3, 2), "max": round(d[-1] / 1e3, 2)}
    t0 = min(r[0] for r in rows)
    out["entry_spread"] = round((max(r[0] for r in rows) - t0) / 1e3, 2)
    out["span"] = round((max(r[7] for r in rows) - t0) / 1e3, 2)
    out["ctas"] = len(rows)
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--case", default="sp_norm", choices=["sp_norm", "prefill", "sample", "decode"])
    ap.add_argument("--batch", type=int, default=6)
    ap.add_argument("--context", type=int, default=1536)
    ap.add_argument("--kv-heads", type=int, default=8)
    ap.add_argument("--trace", action="store_true", help="decode: per-CTA phase trace of one launch")
    ap.add_argument("--world", type=int, default=2)
    ap.add_argument("--tokens", type=int, default=256)
    ap.add_argument("--reps", type=int, default=5)
    args = ap.parse_args()
    peaks = measured_peaks()
    {"sp_norm": case_sp_norm, "prefill": case_prefill, "sample": case_sample,
     "decode": case_decode}[args.case](args, peaks)


if __name__ == "__main__":
    main()
