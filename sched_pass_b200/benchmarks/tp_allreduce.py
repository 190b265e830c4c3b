"""Row-parallel projection + all-reduce: fused sm_100a kernel vs GEMM + NCCL.

Run under torchrun (one rank per GPU). For each decode/prefill shape of the
Llama-3-8B o_proj / down_proj at this TP degree: device time of the fused
kernel and of the baseline (our GEMM followed by NCCL all_reduce) from
CUDA-graph replays (as the engine runs them; eager back-to-back times are
reported beside them), max over ranks, and the fused kernel's fraction of its roofline, where the roofline
time is the slowest of: weight bytes / measured HBM bandwidth, FLOPs /
measured bf16 peak, and bytes this rank must push over NVLink / 770 GB/s.

``--sp`` adds the sequence-parallel sub-layer ("projection + residual add +
RMSNorm, ready for the next GEMM") in its three forms: fused all-reduce +
add_rmsnorm, GEMM + NCCL all-reduce + add_rmsnorm, and GEMM -> reduce-scatter
+ the owner's reduce/norm/all-gather kernel (parallel/sp.py), whose roofline
counts 2 (W-1)/W x T x N x 2 NVLink bytes.
"""
from __future__ import annotations

import argparse
import json
import math
import os

import torch
import torch.distributed as dist

from .. import ops
from ..parallel.tp import TensorParallel, init_distributed
from .common import measured_peaks

NVLINK_GBPS = 770.0  # measured peer copy per direction on this pool


def dev_time(fn, iters=30, warmup=5):
    """ms per call of back-to-back eager launches (includes the host's
    launch cost when that exceeds the kernel), max over ranks."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    dist.barrier()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(iters):
        fn()
    e.record()
    e.synchronize()
    t = torch.tensor([s.elapsed_time(e) / iters], device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t)


def graph_time(fn, iters=30, replays=5):
    """ms per call with `iters` calls (an even number: the fused path's two
    buffer sets alternate in capture order) captured in one CUDA graph and
    replayed -- the device time the engine sees, as its decode steps replay
    graphs. Max over ranks; ranks synchronise between replays."""
    assert iters % 2 == 0
    fn()
    torch.cuda.synchronize()
    dist.barrier()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for _ in range(iters):
            fn()
    torch.cuda.synchronize()
    dist.barrier()
    ts = []
    for _ in range(replays + 1):
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        g.replay()
        e.record()
        e.synchronize()
        ts.append(s.elapsed_time(e) / iters)
        dist.barrier()
    del g  # graphs holding NCCL calls go before the process group
    torch.cuda.synchronize()
    t = torch.tensor([sorted(ts[1:])[len(ts[1:]) // 2]], device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t)


def trace_phases(fn, dev, max_ctas: int = 1024) -> dict:
    """One eager call with the GEMM's per-CTA %globaltimer trace armed.
    Stream-K kernel rows: [entry, fix-up count << 32 | epilogue done (low 32
    bits), after the reduction phase, exit]; cluster kernel rows: [entry, -,
    -, exit]. Returns the phases in us from the earliest CTA entry on this
    rank: when the last CTA finished its own tiles (GEMM + pushes), the
    median and max time CTAs spent in the owned-chunk reduction (flag waits +
    sums), and the last exit."""
    from .._ext import ext
    buf = torch.zeros(max_ctas * 4, dtype=torch.int64, device=dev)
    torch.cuda.synchronize()
    dist.barrier()
    ext().set_gemm_trace(buf.data_ptr())
    try:
        fn()
        torch.cuda.synchronize()
    finally:
        ext().set_gemm_trace(0)
    rows = [[int(v) & ((1 << 64) - 1) for v in r] for r in buf.view(-1, 4).tolist() if r[0] != 0]
    if not rows:
        return {}
    t0 = min(r[0] for r in rows)
    out = {"ctas": len(rows), "exit_us": round((max(r[3] for r in rows) - t0) / 1e3, 2)}
    if max(r[2] for r in rows) != 0:  # stream-K kernel: the epilogue and reduction marks exist
        lo32 = (1 << 32) - 1
        epi = []
        for r in rows:
            e = (r[0] & ~lo32) | (r[1] & lo32)
            epi.append(e + (1 << 32) if e < r[0] else e)
        red = sorted(r[2] - e for r, e in zip(rows, epi))
        out.update({"own_tiles_done_us": round((max(epi) - t0) / 1e3, 2),
                    "reduce_phase_us_p50": round(red[len(red) // 2] / 1e3, 2),
                    "reduce_phase_us_max": round(red[-1] / 1e3, 2),
                    "fixups": sum(r[1] >> 32 for r in rows)})
    return out


def sp_sublayer(args, shapes, world, rank, dev, peaks, fused, base):
    """Row-parallel projection + residual add + RMSNorm, three ways (graph
    replays, max over ranks)."""
    sptp = TensorParallel(mode="sp", device=dev)
    tokens = [int(t) for t in args.tokens.split(",")]
    sp = sptp.sequence_parallel(4096, max(tokens))
    lnw = torch.ones(4096, dtype=torch.bfloat16, device=dev)
    for name, (N, Kfull) in shapes.items():
        K = Kfull // world
        w = (torch.randn(N, K, device=dev) / math.sqrt(Kfull)).to(torch.bfloat16)
        for T in tokens:
            x = torch.randn(T, K, device=dev).to(torch.bfloat16)
            y = torch.empty(T, N, dtype=torch.bfloat16, device=dev)
            res = torch.randn(T, N, device=dev).to(torch.bfloat16)
            normed = torch.empty_like(y)

            def ar_path(tp):
                tp.linear_allreduce(x, w, y)
                ops.add_rmsnorm(y, res, lnw, 1e-5, normed)

            def sp_path():
                sp.linear_rs(x, w)
                _, ready = sp.reduce_norm(res, lnw, 1e-5, T)
                # consume the gathered rows as the next GEMM would (it waits on
                # their ready flags): without it a rank that owns no rows
                # (T < W) is never held back by its peers
                sp.wait_rows(ready, T)

            t_f = graph_time(lambda: ar_path(fused))
            t_b = graph_time(lambda: ar_path(base))
            t_s = graph_time(sp_path)
            t_hbm = N * K * 2 / (peaks["hbm_gbs"] * 1e9)
            t_flop = 2 * T * N * K / (peaks["bf16_tflops"] * 1e12)
            t_nvl = 2 * (world - 1) / world * T * N * 2 / (NVLINK_GBPS * 1e9)
            roof = max(t_hbm, t_flop, t_nvl)
            rec = {"sublayer": name + "+norm", "tp": world, "T": T, "N": N, "K_local": K,
                   "sp_us": round(t_s * 1e3, 2), "fused_ar_us": round(t_f * 1e3, 2),
                   "gemm_nccl_us": round(t_b * 1e3, 2), "sp_vs_fused": round(t_f / t_s, 3),
                   "sp_vs_nccl": round(t_b / t_s, 3), "sp_roofline_us": round(roof * 1e6, 2),
                   "sp_bound": ["hbm", "tensor", "nvlink"][[t_hbm, t_flop, t_nvl].index(roof)],
                   "sp_frac_of_roofline": round(roof * 1e3 / t_s, 3)}
            if rank == 0:
                print(json.dumps(rec), flush=True)
    ops.check_status()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--tokens", default="1,16,64,256,2048")
    ap.add_argument("--sp", action="store_true", help="also time the sequence-parallel sub-layer")
    ap.add_argument("--sp-only", action="store_true")
    ap.add_argument("--trace", action="store_true",
                    help="also report the fused kernel's phases from its per-CTA %%globaltimer trace")
    args = ap.parse_args()
    rank, world, local = init_distributed("nccl")
    dev = torch.device("cuda", local)
    peaks = measured_peaks()
    fused = TensorParallel(mode="fused", device=dev)
    fused.fused_max_bytes = 0  # time the fused kernel at every size
    base = TensorParallel(mode="nccl", device=dev)
    shapes = {"o_proj": (4096, 4096), "down_proj": (4096, 14336)}
    if args.sp or args.sp_only:
        sp_sublayer(args, shapes, world, rank, dev, peaks, fused, base)
    for name, (N, Kfull) in ({} if args.sp_only else shapes).items():
        K = Kfull // world
        w = (torch.randn(N, K, device=dev) / math.sqrt(Kfull)).to(torch.bfloat16)
        for T in (int(t) for t in args.tokens.split(",")):
            x = torch.randn(T, K, device=dev).to(torch.bfloat16)
            y = torch.empty(T, N, dtype=torch.bfloat16, device=dev)
            t_fe = dev_time(lambda: fused.linear_allreduce(x, w, y))
            t_be = dev_time(lambda: base.linear_allreduce(x, w, y))
            t_f = graph_time(lambda: fused.linear_allreduce(x, w, y))
            t_b = graph_time(lambda: base.linear_allreduce(x, w, y))
            t_g = graph_time(lambda: ops.linear(x, w, y))  # the GEMM alone (no collective)
            phases = trace_phases(lambda: fused.linear_allreduce(x, w, y), dev) if args.trace else None
            wbytes = N * K * 2
            t_hbm = wbytes / (peaks["hbm_gbs"] * 1e9)
            t_flop = 2 * T * N * K / (peaks["bf16_tflops"] * 1e12)
            t_nvl = (world - 1) * T * N * 2 / (NVLINK_GBPS * 1e9)
            roof = max(t_hbm, t_flop, t_nvl)
            rec = {"op": name, "tp": world, "T": T, "N": N, "K_local": K,
                   "fused_us": round(t_f * 1e3, 2), "gemm_plus_nccl_us": round(t_b * 1e3, 2),
                   "gemm_only_us": round(t_g * 1e3, 2), "collective_share_us": round((t_f - t_g) * 1e3, 2),
                   "eager_fused_us": round(t_fe * 1e3, 2), "eager_gemm_plus_nccl_us": round(t_be * 1e3, 2),
                   "speedup": round(t_b / t_f, 3), "roofline_us": round(roof * 1e6, 2),
                   "oneshot_push_bytes": (world - 1) * T * N * 2,
                   "bound": ["hbm", "tensor", "nvlink"][[t_hbm, t_flop, t_nvl].index(roof)],
                   "frac_of_roofline": round(roof * 1e3 / t_f, 3)}
            if phases is not None:
                ph = [None] * world
                dist.all_gather_object(ph, phases)
                rec["phases_by_rank"] = ph
            if rank == 0:
                print(json.dumps(rec), flush=True)
    ops.check_status()
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
