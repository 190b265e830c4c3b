#!/usr/bin/env python
"""One Mixtral MoE layer on one GPU (all experts local): router -> dispatch
-> fp8 gate/up expert GEMM -> activation quantisation -> fp8 down expert GEMM
with the combine epilogue -> combine + residual + RMSNorm.

Reports the CUDA-event time of the whole layer (median of ``--iters`` after
``--warmup``; the expert weights, 1.4 GB for Mixtral-8x7B, exceed L2, so no
flush is needed) and the achieved fraction of the measured HBM bandwidth for
the bytes the layer must read: the weights of every expert that received a
token plus the activations.

    python -m sched_pass_b200.benchmarks.moe_layer --tokens 128

``--hot FRAC`` sends a fraction of the tokens to expert 0 (a shared component
along its router row: the reference's hot-expert imbalance experiment), and
``--capacity-factor CF`` caps every expert at CF x tokens x top_k / experts
rows (the E2 capacity lever; the overflow is dropped and counted).
"""
from __future__ import annotations

import argparse
import json

import torch


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="mixtral-8x7b")
    ap.add_argument("--tokens", type=int, default=128)
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--hot", type=float, default=0.0, help="fraction of tokens routed to expert 0")
    ap.add_argument("--capacity-factor", type=float, default=0.0, help="0: no cap")
    args = ap.parse_args(argv)

    from sched_pass_b200 import ops
    from sched_pass_b200.benchmarks.common import measured_peaks
    from sched_pass_b200.models.config import get_config
    from sched_pass_b200.parallel.ep import ExpertParallel, build_moe_weights

    cfg = get_config(args.model)
    dev = torch.device("cuda", 0)
    T = args.tokens
    cap = None
    if args.capacity_factor > 0:
        cap = max(1, int(args.capacity_factor * T * cfg.top_k / cfg.n_experts))
    ep = ExpertParallel(cfg, dev, max_tokens=max(T, 1), capacity=cap)
    g = torch.Generator(device=dev).manual_seed(0)
    w = build_moe_weights(cfg, 0, 1, g, dev)
    x = torch.randn(T, cfg.hidden, device=dev, generator=g)
    n_hot = int(args.hot * T)
    if n_hot:
        r0 = w.router[0].float()
        x[:n_hot] += 8.0 * r0 / r0.norm()  # +8 on expert 0's logit (others ~ N(0, 1))
    x = x.to(torch.bfloat16)
    h = torch.randn(T, cfg.hidden, device=dev, generator=g).to(torch.bfloat16)
    y = torch.empty_like(x)
    ln = torch.ones(cfg.hidden, dtype=torch.bfloat16, device=dev)
    for _ in range(args.warmup):
        ep.layer(w, x, h, ln, y, cfg.rms_eps)
    torch.cuda.synchronize()
    ops.check_status()
    times = []
    for _ in range(args.iters):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        ep.layer(w, x, h, ln, y, cfg.rms_eps)
        e1.record()
        e1.synchronize()
        times.append(e0.elapsed_time(e1) * 1e3)
    ops.check_status()
    times.sort()
    us = times[len(times) // 2]
    active = int((ep.words[: ep.E_local] > 0).sum().item())  # rows_valid of the last call
    H, I = cfg.hidden, cfg.ffn
    wbytes = active * (2 * I * H + H * I)
    abytes = T * cfg.top_k * (H + 2 * I + I + 2 * H)
    peaks = measured_peaks()
    hbm = peaks.get("hbm_gbs", 6650.0)
    out = {"kernel": "moe_layer", "model": cfg.name, "tokens": T, "experts_active": active,
           "hot": args.hot, "capacity": cap, "dropped": ep.dropped_total(),
           "rows_per_expert": [int(v) for v in ep.words[: ep.E_local].tolist()],
           "us_median": round(us, 2), "us_min": round(times[0], 2),
           "bytes": wbytes + abytes, "achieved_gbs": round((wbytes + abytes) / us / 1e3, 1),
           "frac_of_measured_hbm": round((wbytes + abytes) / us / 1e3 / hbm, 3)}
    print(json.dumps(out))
    ep.close()
    return out


if __name__ == "__main__":
    main()
