#!/usr/bin/env python
"""Mixtral-8x7B-architecture MoE decode with expert parallelism over N GPUs.

Workload (the named config): decode batch 128 in total, a context of 3072
random tokens per request, 128 output tokens; 32 layers, hidden 4096,
32 query / 8 KV heads, 8 experts top-2, expert FFN 14336, experts stored as
fp8 e4m3 with 128x128 block scales. Attention runs data-parallel (each rank
serves batch / N requests with replicated attention weights), the experts are
split across the N ranks and every MoE layer is the fused NVLink dispatch ->
grouped fp8 expert GEMMs -> combine of ``parallel/ep.py``.

The contexts are synthetic: every KV page is filled with N(0, 1) values and
the requests join the decode set directly (``Engine.add_prefilled``); decode
cost does not depend on the values in the cache. ``--prefill real`` runs the
prompts through the engine's chunked prefill instead.

Timing: W warm-up decode steps (CUDA-graph capture included), then K steps
between barriers and device synchronisations, CUDA events on the engine
stream, max over ranks. Every step streams >5 GB of weights and KV per GPU,
far above L2, so no flush is needed.

Run: ``python -m torch.distributed.run --nproc-per-node N --master-addr
127.0.0.1 -m sched_pass_b200.benchmarks.mixtral_decode --gpus N``.
"""
from __future__ import annotations

import argparse
import json
import os
import time

import numpy as np
import torch
import torch.distributed as dist


def parse(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--model", default="mixtral-8x7b")
    ap.add_argument("--batch", type=int, default=128, help="decode batch over all ranks")
    ap.add_argument("--context", type=int, default=3072)
    ap.add_argument("--output", type=int, default=128)
    ap.add_argument("--steps", type=int, default=60)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--prefill", default="synthetic", choices=["synthetic", "real"])
    ap.add_argument("--acquire", default="auto", choices=["static", "ticket", "clc", "auto"])
    ap.add_argument("--no-graphs", action="store_true")
    ap.add_argument("--seed", type=int, default=0)
    return ap.parse_args(argv)


def main(argv=None):
    args = parse(argv)
    from sched_pass_b200.engine.engine import Engine, EngineConfig
    from sched_pass_b200.engine.request import Request
    from sched_pass_b200.models.config import get_config
    from sched_pass_b200.models.mixtral import mixtral_factory
    from sched_pass_b200.parallel.ep import ExpertParallel
    from sched_pass_b200.parallel.tp import init_distributed
    from sched_pass_b200.utils.clocks import ClockSampler

    rank, world, local = init_distributed("nccl", timeout_s=300)
    assert world == args.gpus, f"--gpus {args.gpus} but WORLD_SIZE {world}"
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    cfg = get_config(args.model)
    assert args.batch % world == 0
    B = args.batch // world
    max_ctx = (args.context + args.output + 16 + 127) // 128 * 128
    prefill_tokens = 4096 if args.prefill == "real" else 256
    ecfg = EngineConfig(max_batch=B, max_prefill_tokens=prefill_tokens, max_context=max_ctx,
                        cuda_graphs=not args.no_graphs, levers=True, acquire=args.acquire, seed=args.seed)
    T = max(ecfg.max_prefill_tokens + ecfg.max_batch, 256)
    ep = ExpertParallel(cfg, dev, max_tokens=T)
    eng = Engine(cfg, ecfg, dev, model_factory=mixtral_factory(ep, rank, world))

    rng = np.random.default_rng(args.seed + rank)
    prompts = rng.integers(0, cfg.vocab, size=(B, args.context), dtype=np.int64).astype(np.int32)
    reqs = [Request(rid=i, prompt=prompts[i], max_new_tokens=args.output, urgency=float(rng.random()))
            for i in range(B)]
    if args.prefill == "synthetic":
        eng.fill_kv_random(args.seed + 17 * rank)
        for r in reqs:
            eng.add_prefilled(r, int(rng.integers(0, cfg.vocab)))
    else:
        for r in reqs:
            eng.add_request(r)
        # every rank has the same prompt lengths, so the same number of steps
        while any(r.state.name != "DECODE" for r in reqs):
            eng.step()
    steps_left = min(r.max_new_tokens - len(r.output) for r in reqs)
    if args.warmup + args.steps > steps_left:
        raise SystemExit(f"--warmup + --steps must be <= {steps_left} decode steps of this workload")
    for _ in range(args.warmup):
        eng.step()

    stream = torch.cuda.current_stream(dev)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    vis = os.environ.get("CUDA_VISIBLE_DEVICES", "")
    parts = vis.split(",") if vis else []
    phys = int(parts[local]) if len(parts) > local and parts[local].isdigit() else local
    sampler = ClockSampler(gpu_index=phys).start()
    first = len(eng.stats)
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    t0 = time.perf_counter()
    ev0.record(stream)
    tokens = 0
    for _ in range(args.steps):
        plan, _ = eng.step()
        tokens += len(plan.decode)
    ev1.record(stream)
    torch.cuda.synchronize(dev)
    t1 = time.perf_counter()
    if world > 1:
        dist.barrier()
    clocks = sampler.stop()
    dev_s, host_s = ev0.elapsed_time(ev1) / 1e3, t1 - t0
    kernel_ms = float(np.sum([s.device_ms for s in eng.stats[first:]]))
    tok = torch.tensor([dev_s, host_s, kernel_ms, tokens, ep.dropped_total()], dtype=torch.float64, device=dev)
    if world > 1:
        mx = tok.clone()
        dist.all_reduce(mx, op=dist.ReduceOp.MAX)
        sm = tok.clone()
        dist.all_reduce(sm, op=dist.ReduceOp.SUM)
        dev_s, host_s, kernel_ms = float(mx[0]), float(mx[1]), float(mx[2])
        tokens, dropped = int(sm[3]), int(sm[4])
    else:
        dropped = int(tok[4])
    step_ms = sorted(s.device_ms for s in eng.stats[first:])
    per_layer = 10  # qkv+rope gemm, attention, o gemm, add+norm, router, dispatch, 2 expert gemms, quantize, combine+norm
    out = {
        "metric": "decode tokens/s (Mixtral-8x7B-arch, EP)",
        "value": round(tokens / dev_s, 2),
        "unit": "decode tokens/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(1e3 * dev_s / args.steps, 4),
        "kernel_ms_per_step_max_rank": round(kernel_ms / args.steps, 4),
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "fp8 e4m3 experts (128x128 block scales), bf16 attention/activations",
        "data": ("synthetic: random token ids, random-init weights, "
                 + ("N(0,1) KV for the 3072-token contexts (no prefill)" if args.prefill == "synthetic"
                    else "contexts prefilled by the engine")),
        "config": {"model": cfg.name + "-arch", "global_batch": args.batch, "seq_len": args.context,
                   "output_tokens": args.output, "parallelism": f"ep{world} (attention dp{world})",
                   "l2": "inputs larger than L2 (weights and KV stream every step)"},
        "step_ms_p50": round(step_ms[len(step_ms) // 2], 3),
        "step_ms_p99": round(step_ms[min(len(step_ms) - 1, int(0.99 * len(step_ms)))], 3),
        "dropped_assignments": dropped,
        "e2e": {"value": round(tokens / host_s, 2), "unit": "decode tokens/s",
                "h2d_bytes_per_step": eng.packed_len * 4, "d2h_bytes_per_step": 4 * B},
        "gpu_launches": int(args.steps * (cfg.n_layers * per_layer + 4)),
        "clocks": clocks,
    }
    if rank == 0:
        print(json.dumps(out))
    if world > 1:
        dist.barrier()
    eng.graphs.clear()
    ep.close()
    if world > 1:
        dist.destroy_process_group()
    return out


if __name__ == "__main__":
    main()
