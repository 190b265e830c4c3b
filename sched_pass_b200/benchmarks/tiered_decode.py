#!/usr/bin/env python
"""Long-context tiered-KV decode: Llama-3-70B architecture, tensor parallel.

Workload (the named config): 64 concurrent requests with contexts uniform in
[32768, 131072] tokens and 256 output tokens, TP over N GPUs, random-init
bf16 weights. The KV that does not fit in the device pool spills to pinned
host memory (engine/tiered_kv.py); every step streams the host pages it
reads back one layer at a time through the copy kernel, overlapped with the
previous layer's compute. Shed budgets (tau = 0.5 x context) go to the
25% least urgent requests -- their pages beyond tau are the first to spill
and are never read again -- and cluster launch control is armed only when
the cost estimator is uncertain (acquire=auto).

The contexts are synthetic: KV pages hold N(0, 1) values and the requests
join the decode set directly (``Engine.add_prefilled``). Sizes scale with
``--requests`` / ``--ctx-min`` / ``--ctx-max`` for smaller boxes; the JSON
line reports the sizes used and the device / host / staged page counts.

Run: ``python -m torch.distributed.run --nproc-per-node 8 --master-addr
127.0.0.1 -m sched_pass_b200.benchmarks.tiered_decode --gpus 8``.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import time

import numpy as np
import torch
import torch.distributed as dist


def parse(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--model", default="llama-3-70b")
    ap.add_argument("--requests", type=int, default=64)
    ap.add_argument("--ctx-min", type=int, default=32768)
    ap.add_argument("--ctx-max", type=int, default=131072)
    ap.add_argument("--output", type=int, default=256)
    ap.add_argument("--steps", type=int, default=8)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--shed-fraction", type=float, default=0.25)
    ap.add_argument("--shed-ratio", type=float, default=0.5)
    ap.add_argument("--device-kv-gb", type=float, default=0.0, help="cap of the device KV pool (0: what fits)")
    ap.add_argument("--acquire", default="auto")
    ap.add_argument("--host-kv-dtype", default="bf16", choices=["bf16", "fp8"],
                    help="host pool storage; fp8 halves the bytes staged over PCIe")
    ap.add_argument("--seed", type=int, default=0)
    return ap.parse_args(argv)


def main(argv=None):
    args = parse(argv)
    from sched_pass_b200.engine.engine import Engine, EngineConfig
    from sched_pass_b200.engine.request import Request
    from sched_pass_b200.models.config import get_config
    from sched_pass_b200.parallel.tp import TensorParallel, init_distributed
    from sched_pass_b200.utils.clocks import ClockSampler

    rank, world, local = init_distributed("nccl", timeout_s=600)
    assert world == args.gpus
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    tp = TensorParallel(device=dev) if world > 1 else None
    cfg = get_config(args.model)
    hkv = cfg.n_kv_heads // world
    page_bytes = 2 * cfg.n_layers * hkv * 16 * cfg.head_dim * 2
    rng = np.random.default_rng(args.seed)
    ctx = rng.integers(args.ctx_min, args.ctx_max + 1, size=args.requests)
    need_pages = int(sum(math.ceil((c + args.output) / 16) for c in ctx))
    # device budget: what is free after the weights, minus a margin
    free, _ = torch.cuda.mem_get_info(dev)
    weights = cfg.param_count() * 2 // world
    budget = free - weights - 12 * (1 << 30)
    if args.device_kv_gb > 0:
        budget = min(budget, int(args.device_kv_gb * (1 << 30)))
    # staging holds one layer of every host page a step may read, twice
    # (even / odd layers): 2 / layers of a page per slot
    slot_bytes = 2 * page_bytes // cfg.n_layers
    alloc_pages = max(64, budget // page_bytes)
    for _ in range(4):  # settle the split between resident pages and staging slots
        host_pages = max(16, need_pages - alloc_pages + 64)
        alloc_pages = max(64, (budget - host_pages * slot_bytes) // page_bytes)
    host_pages = max(16, need_pages - alloc_pages + 64)
    staging = host_pages
    max_ctx = int(ctx.max()) + args.output + 16
    ecfg = EngineConfig(max_batch=args.requests, max_prefill_tokens=256,
                        max_context=(max_ctx + 127) // 128 * 128, num_pages=alloc_pages,
                        host_kv_pages=host_pages, kv_staging_pages=staging, host_kv_dtype=args.host_kv_dtype,
                        acquire=args.acquire,
                        shed_fraction=args.shed_fraction, shed_ratio=args.shed_ratio, seed=args.seed)
    eng = Engine(cfg, ecfg, dev, tp=tp)
    g = torch.Generator(device=dev)
    g.manual_seed(args.seed + 1)
    eng.kv.k.normal_(generator=g)
    eng.kv.v.normal_(generator=g)
    urg = rng.random(args.requests)
    low = set(np.argsort(urg)[: int(args.shed_fraction * args.requests)].tolist())
    reqs = []
    for i in range(args.requests):
        r = Request(rid=i, prompt=rng.integers(0, cfg.vocab, size=int(ctx[i])).astype(np.int32),
                    max_new_tokens=args.output, urgency=float(urg[i]),
                    tau=int(args.shed_ratio * ctx[i]) if i in low else 0)
        eng.add_prefilled(r, int(rng.integers(0, cfg.vocab)))
        reqs.append(r)
    torch.cuda.synchronize(dev)
    for _ in range(args.warmup):
        eng.step()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    sampler = ClockSampler(gpu_index=local).start()
    stream = torch.cuda.current_stream(dev)
    staged0 = eng.tier.staged_pages
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0 = time.perf_counter()
    e0.record(stream)
    tokens = 0
    for _ in range(args.steps):
        plan, _ = eng.step()
        tokens += len(plan.decode)
    e1.record(stream)
    torch.cuda.synchronize(dev)
    t1 = time.perf_counter()
    if world > 1:
        dist.barrier()
    clocks = sampler.stop()
    t = torch.tensor([e0.elapsed_time(e1) / 1e3, t1 - t0], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    dev_s, host_s = float(t[0]), float(t[1])
    staged = (eng.tier.staged_pages - staged0) / max(1, args.steps)
    out = {
        "metric": f"decode tokens/s ({cfg.name}-arch, tiered KV)",
        "value": round(tokens / dev_s, 3), "unit": "decode tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(1e3 * dev_s / args.steps, 3),
        "tpot_ms": round(1e3 * dev_s / args.steps, 3), "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic: random token ids, random-init weights, N(0,1) KV (no prefill)",
        "config": {"model": cfg.name + "-arch", "requests": args.requests,
                   "context": [args.ctx_min, args.ctx_max], "output_tokens": args.output,
                   "parallelism": f"tp{world}", "shed": f"{args.shed_fraction} least urgent, tau={args.shed_ratio}x",
                   "acquire": args.acquire, "host_kv_dtype": args.host_kv_dtype},
        "kv": {"pages_needed": need_pages, "device_pages": alloc_pages, "staging_pages": staging,
               "host_pages": host_pages, "spilled_pages": eng.tier.spilled_pages,
               "staged_pages_per_step": round(staged, 1),
               "staged_gb_per_step": round(staged * page_bytes / (2 if args.host_kv_dtype == "fp8" else 1) / 1e9,
                                           3)},
        "e2e": {"value": round(tokens / host_s, 3), "unit": "decode tokens/s",
                "h2d_bytes_per_step": eng.packed_len * 4, "d2h_bytes_per_step": 4 * args.requests},
        "clocks": clocks,
    }
    if rank == 0:
        print(json.dumps(out))
    if world > 1:
        dist.barrier()
    eng.graphs.clear()
    if world > 1:
        dist.destroy_process_group()
    return out


if __name__ == "__main__":
    main()
