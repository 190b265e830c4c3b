"""torchrun worker: the fused GEMM + all-reduce's low-latency exchange with
NVLink multicast line buffers (one multimem store per line) against the same
exchange over per-peer stores: bit-identical outputs, and the per-call device
time of each (CUDA graph of back-to-back calls, max over ranks)."""
import faulthandler
import json
import math
import os
import sys

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))))

from sched_pass_b200 import ops  # noqa: E402
from sched_pass_b200.parallel.fused import FusedAllReduce  # noqa: E402
from sched_pass_b200.parallel.tp import init_distributed  # noqa: E402

faulthandler.enable()

CALLS = 20  # per graph (even: the flag path's slab sets alternate; the line path keeps its epoch on the device)


def graph_us(fn, reps=5):
    """Per-call device time of CALLS back-to-back calls captured in one CUDA
    graph, median of `reps` replays; every rank replays together."""
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for _ in range(3):
            fn()
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for _ in range(CALLS):
            fn()
    times = []
    for _ in range(reps + 1):
        dist.barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        g.replay()
        e1.record()
        torch.cuda.synchronize()
        times.append(e0.elapsed_time(e1) * 1e3 / CALLS)
    del g
    t = sorted(times[1:])[len(times[1:]) // 2]
    v = torch.tensor([t], device="cuda")
    dist.all_reduce(v, op=dist.ReduceOp.MAX)
    return float(v.item())


def main():
    rank, world, local = init_distributed("nccl", timeout_s=60)
    dev = torch.device("cuda", local)
    os.environ["SCHED_TP_NVLS"] = "0"
    peer = FusedAllReduce(None, dev, max_tokens=64, max_n=8192)
    os.environ["SCHED_TP_NVLS"] = "1"
    mc = FusedAllReduce(None, dev, max_tokens=64, max_n=8192)
    out = {"world": world, "multicast": bool(mc.ll_mc), "checks": []}
    print(f"STAGE {rank} buffers ready (multicast {bool(mc.ll_mc)})", flush=True)
    g = torch.Generator(device="cpu").manual_seed(7)
    try:
        run_checks(rank, world, dev, peer, mc, g, out)
    except Exception as e:  # recorded; every rank still reaches the common teardown below
        out["error"] = f"rank {rank}: {type(e).__name__}: {e}"
        print(f"STAGE {rank} error {out['error']}", flush=True)
    dist.barrier()
    peer.close()
    mc.close()
    errs = [None] * world
    dist.all_gather_object(errs, out.get("error"))
    out["errors"] = [x for x in errs if x]
    if rank == 0:
        print("NVLSJSON " + json.dumps(out), flush=True)
    dist.barrier()
    dist.destroy_process_group()


def run_checks(rank, world, dev, peer, mc, g, out):
    # (T, N, K per rank): Llama-3-8B o_proj at TP=world is N = 4096, K = 4096 / world
    for (T, N, K) in [(1, 4096, 4096 // world), (16, 4096, 4096 // world), (32, 4096, 14336 // world)]:
        x_full = torch.randn(T, K * world, generator=g)
        w_full = torch.randn(N, K * world, generator=g) / math.sqrt(K * world)
        ref = x_full.to(torch.bfloat16).float() @ w_full.to(torch.bfloat16).float().t()
        x = x_full[:, rank * K:(rank + 1) * K].to(torch.bfloat16).to(dev).contiguous()
        w = w_full[:, rank * K:(rank + 1) * K].to(torch.bfloat16).to(dev).contiguous()
        y0 = torch.empty(T, N, dtype=torch.bfloat16, device=dev)
        y1 = torch.empty_like(y0)
        for _ in range(3):
            peer.linear_allreduce(x, w, y0)
            mc.linear_allreduce(x, w, y1)
        torch.cuda.synchronize()
        ops.check_status()
        exact = bool(torch.equal(y0, y1))
        err = ((y1.float().cpu() - ref).norm() / ref.norm()).item()
        us_peer = graph_us(lambda: peer.linear_allreduce(x, w, y0))
        us_mc = graph_us(lambda: mc.linear_allreduce(x, w, y1))
        torch.cuda.synchronize()
        ops.check_status()
        exact_after = bool(torch.equal(y0, y1))
        out["checks"].append({"T": T, "N": N, "K": K, "bit_exact": exact and exact_after, "rel_err": err,
                              "us_peer_stores": round(us_peer, 2), "us_multicast": round(us_mc, 2)})
        print(f"STAGE {rank} T={T} done", flush=True)


if __name__ == "__main__":
    main()
