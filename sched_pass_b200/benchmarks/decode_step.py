"""Steady decode steps of the engine at a fixed batch and context.

Fills ``--batch`` requests with ``--context``-token prompts (through the
engine's prefill), then times decode steps (CUDA-graph replay unless
``--no-graphs``). Prints per-step device time, tokens/s, and the implied
weight-streaming bandwidth. ``--profile-steps N`` wraps N eager decode steps
in an NVTX range named ``profile_step`` so a profiler can select exactly
those kernels.
"""
from __future__ import annotations

import argparse
import json

import numpy as np
import torch

from .. import ops
from ..engine.engine import Engine, EngineConfig
from ..engine.request import Request
from ..models.config import get_config
from .common import measured_peaks


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="llama-3-8b")
    ap.add_argument("--batch", type=int, default=16)
    ap.add_argument("--context", type=int, default=1536)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--acquire", default="static")
    ap.add_argument("--levers", type=int, default=1)
    ap.add_argument("--no-graphs", action="store_true")
    ap.add_argument("--profile-steps", type=int, default=0)
    ap.add_argument("--target-tasks", type=int, default=0,
                    help="decode-attention tasks to aim for when splitting KV (0: one per SM)")
    args = ap.parse_args()
    cfg = get_config(args.model)
    new_tokens = args.steps + args.profile_steps + 8
    ecfg = EngineConfig(max_batch=max(args.batch, 8), max_prefill_tokens=4096,
                        max_context=(args.context + new_tokens + 127) // 128 * 128,
                        cuda_graphs=not args.no_graphs, levers=bool(args.levers), acquire=args.acquire,
                        target_tasks=args.target_tasks)
    eng = Engine(cfg, ecfg, "cuda")
    rng = np.random.default_rng(0)
    for i in range(args.batch):
        eng.add_request(Request(rid=i, prompt=rng.integers(0, cfg.vocab, size=args.context).astype(np.int32),
                                max_new_tokens=new_tokens))
    # prefill until every request decodes
    while any(len(r.output) == 0 for r in eng.sched.running) or eng.sched.waiting:
        eng.step()
    for _ in range(3):
        eng.step()
    torch.cuda.synchronize()
    if args.profile_steps:
        eng.ecfg.cuda_graphs = False
        torch.cuda.nvtx.range_push("profile_step")
        for _ in range(args.profile_steps):
            eng.step()
        torch.cuda.synchronize()
        torch.cuda.nvtx.range_pop()
        eng.ecfg.cuda_graphs = not args.no_graphs
    n0 = len(eng.stats)
    for _ in range(args.steps):
        eng.step()
    ms = [s.device_ms for s in eng.stats[n0:]]
    ops.check_status()
    med = float(np.median(ms))
    wbytes = sum(t.numel() * t.element_size() for t in
                 [eng.model.w.lm_head] + [x for lw in eng.model.w.layers for x in (lw.qkv, lw.o, lw.gate_up, lw.down)])
    kvbytes = args.batch * (args.context + 8) * cfg.kv_bytes_per_token()
    print(json.dumps({"batch": args.batch, "context": args.context, "splits": eng.splits_for(args.batch),
                      "step_ms_p50": round(med, 4),
                      "step_ms_min": round(min(ms), 4), "tok_s": round(args.batch / med * 1e3, 1),
                      "weights_GB": round(wbytes / 1e9, 2), "kv_GB": round(kvbytes / 1e9, 3),
                      "effective_GBps": round((wbytes + kvbytes) / med / 1e6, 1),
                      "frac_hbm_of_measured": round((wbytes + kvbytes) / med / 1e6 / measured_peaks()["hbm_gbs"], 3),
                      "graphs": not args.no_graphs}))


if __name__ == "__main__":
    main()
