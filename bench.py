#!/usr/bin/env python
"""Decode-serving benchmark: Llama-3-8B architecture, tensor parallel over N GPUs.

Workload (the named config): synthetic requests with Poisson arrivals at
8 req/s, 1536 random prompt tokens, 128 output tokens, continuous batching,
all scheduling levers armed every step. Random-initialised bf16 weights.

Steady-state window. The engine's own scheduler is first driven through the
workload without the model on a nominal step clock
(``benchmarks/steady_state.py``) to pick the most representative window of
W + K steps after ``--horizon`` seconds of workload, and is then replayed to
the window's start (the requests in flight hold synthetic KV). The W warm-up
and K timed steps run the model; their admissions follow the same nominal
clock, so every GPU count serves exactly the same requests, batch sizes and
prefill chunks (a fixed load: strong scaling). Arrivals inside the window are
prefilled inside the timed region. Decode-step CUDA graphs for the window's
batch sizes and one prefill-sized eager step run before timing.

The K steps are timed between two barriers + synchronisations with CUDA
events on the engine's stream (max over ranks); an event at every step start
gives each step's duration (max over ranks), from which every request's
inter-token intervals inside the window are formed.

Reported:
  value        decode tokens / s of the timed steps (device time)
  p50/p99 TPOT per-request mean inter-token interval inside the window
               (every request that produced two tokens in it), and the p50 /
               p99 of all inter-token intervals
  e2e.value    the same tokens over the host clock of the same loop, which
               includes each step's pinned H2D input copy and the D2H read of
               the sampled tokens through ``Engine.step_async`` / ``drain``
               (the public API; the host plans step k while the device runs
               step k - 1)
  gpu_launches kernel launches of this framework's extension in the timed
               steps (counted at the launchers; a replayed graph adds the
               launches it captured)
Weights (16 GB at TP=1) stream from HBM every step, more than L2 holds, so
no flush is needed between steps.

``--impl reference`` would run the reference project (jc-su/sched-pass)
through its own public API; it cannot be installed or run here (see
``reference_arm``), so that arm prints an ``unavailable`` line.
"""
from __future__ import annotations

import argparse
import gc
import json
import math
import os
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

BASELINE_VALUE = None  # the reference publishes no number for this metric/config
METRIC = "decode tokens/sec/box and p99 TPOT at 1/2/4/8 B200 vs reference NCCL build"


def parse(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--model", default="llama-3-8b")
    ap.add_argument("--rate", type=float, default=8.0)
    ap.add_argument("--prompt", type=int, default=1536)
    ap.add_argument("--output", type=int, default=128)
    ap.add_argument("--requests", type=int, default=2000)
    ap.add_argument("--max-batch", type=int, default=128)
    ap.add_argument("--horizon", type=float, default=30.0,
                    help="workload seconds before the earliest window start (start-up transient)")
    ap.add_argument("--search", type=float, default=60.0,
                    help="workload seconds after the horizon in which the window is chosen")
    ap.add_argument("--nominal-step-ms", type=float, default=None,
                    help="nominal decode step of the admission clock (default: the 1-GPU figure)")
    ap.add_argument("--nominal-prefill-us", type=float, default=None,
                    help="nominal time per prefill token of the admission clock")
    ap.add_argument("--step-tokens", type=int, default=0,
                    help="cap on decode + prefill tokens per engine step (0: prefill chunks up to 2048)")
    ap.add_argument("--acquire", default="auto", choices=["static", "ticket", "clc", "auto"])
    ap.add_argument("--tp-mode", default=None, choices=[None, "fused", "nccl", "sp"])
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--no-graphs", action="store_true")
    return ap.parse_args(argv)


def reference_arm(args):
    """The reference's serving path is SGLang + FlashInfer with its LLVM pass
    plugin woven in by clang (jc-su/sched-pass SGLANG.md, scripts/bench_ab.sh).
    pip cannot install it (no setup.py or pyproject.toml), and this image has
    neither SGLang nor clang/LLVM development files, so nothing of its stock
    code path can run: print the unavailable line."""
    ref = os.path.join(ROOT, "baseline", "_ref")
    missing = [m for m in ("sglang",) if not _importable(m)]
    why = ("reference not installable offline: jc-su/sched-pass has no setup.py/pyproject.toml "
           "(pip: 'not installable'), and its serving path needs clang+LLVM for the pass plugin and "
           f"SGLang ({', '.join(missing) or 'present'} missing in this image)")
    if os.path.isdir(ref) and os.listdir(ref):
        why = "reference install present but its serving path needs clang+LLVM and SGLang (absent)"
    print(json.dumps({"impl": "reference", "unavailable": why}))
    return 0


def _importable(name: str) -> bool:
    import importlib.util
    return importlib.util.find_spec(name) is not None


def pct(v, p):
    """Nearest-rank percentile of an ascending list (None if empty)."""
    if not v:
        return None
    return float(v[min(len(v) - 1, max(0, int(math.ceil(p / 100.0 * len(v))) - 1))])


def window_tpot(produced: list, step_s: list) -> dict:
    """Inter-token statistics of a window. ``produced[i]`` lists the request
    ids that produced a token at timed step i (index -1: the step before the
    window); ``step_s[i]`` is step i's duration. An interval counts when both
    of its tokens came from steps >= -1, so it lies wholly in the window."""
    start = np.concatenate([[0.0], np.cumsum(step_s)])  # time at which step i ends = start[i + 1]
    last = {rid: -1 for rid in produced[0]}
    itl, per_req = [], {}
    for i, rids in enumerate(produced[1:]):
        t = start[i + 1]
        for rid in rids:
            j = last.get(rid)
            if j is not None:
                dt = t - (start[j + 1] if j >= 0 else 0.0)
                itl.append(dt)
                per_req.setdefault(rid, []).append(dt)
            last[rid] = i
    tpot = sorted(float(np.mean(v)) for v in per_req.values())
    itl.sort()
    return {"tpot": tpot, "itl": itl, "requests": len(per_req)}


def main(argv=None):
    args = parse(argv)
    if args.impl == "reference":
        return reference_arm(args)

    import torch
    import torch.distributed as dist

    from sched_pass_b200 import _ext
    from sched_pass_b200.benchmarks import steady_state as ss
    from sched_pass_b200.engine.engine import Engine, EngineConfig
    from sched_pass_b200.engine.request import Request
    from sched_pass_b200.models.config import get_config
    from sched_pass_b200.parallel.tp import TensorParallel, init_distributed
    from sched_pass_b200.utils.clocks import ClockSampler

    rank, world, local = init_distributed("nccl")
    assert world == args.gpus, f"--gpus {args.gpus} but WORLD_SIZE {world}"
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    tp = TensorParallel(mode=args.tp_mode, device=dev) if world > 1 else None
    cfg = get_config(args.model)
    max_ctx = args.prompt + args.output + 16
    ecfg = EngineConfig(max_batch=args.max_batch, max_prefill_tokens=2048, max_step_tokens=args.step_tokens,
                        max_context=(max_ctx + 127) // 128 * 128, cuda_graphs=not args.no_graphs,
                        levers=True, acquire=args.acquire, seed=args.seed, clock_sync=False)
    eng = Engine(cfg, ecfg, dev, tp=tp)

    # workload: the same on every rank (same seed)
    rng = np.random.default_rng(args.seed)
    arrivals = np.cumsum(rng.exponential(1.0 / args.rate, size=args.requests))
    prompts = rng.integers(0, cfg.vocab, size=(args.requests, args.prompt), dtype=np.int64).astype(np.int32)
    reqs = [Request(rid=i, prompt=prompts[i], max_new_tokens=args.output, arrival=float(arrivals[i]),
                    urgency=float(rng.random())) for i in range(args.requests)]
    step_s = (args.nominal_step_ms or ss.NOMINAL_DECODE_STEP_S * 1e3) / 1e3
    tok_s = (args.nominal_prefill_us or ss.NOMINAL_PREFILL_TOKEN_S * 1e6) / 1e6
    cost = lambda nd, npf: ss.nominal_cost(nd, npf, step_s, tok_s)  # noqa: E731

    # 1. the window: simulate the scheduler, pick the most representative start
    trace = ss.simulate(eng.new_scheduler, reqs, cfg.vocab, args.horizon + args.search, cost)
    s0, window = ss.pick_window(trace, args.steps, args.warmup, args.horizon)

    # 2. kernels warm before any timing: one prefill-sized eager step (two
    # dummy prompts filling the 2048-token budget), aborted afterwards, and
    # the decode graphs of every batch size the warm-up and timed steps see
    dummies = [Request(rid=-1 - i, prompt=prompts[i][:n].copy(), max_new_tokens=2)
               for i, n in enumerate((args.prompt, max(16, ecfg.max_prefill_tokens - args.prompt)))]
    for d in dummies:
        eng.add_request(d)
    eng.step()
    for d in dummies:
        eng.abort(d)
    eng.warm_decode_graphs(trace.n_decode[s0:s0 + args.warmup + args.steps].tolist())
    eng.fill_kv_random(args.seed)

    # 3. replay the scheduler to the window's start, then the warm-up steps
    drv = ss.replay(eng.sched, reqs, cfg.vocab, s0, cost)
    eng.clock = drv.clock
    last_producers = []

    def one_step():
        drv.admit(eng.add_request)
        if not eng.has_work():
            return None
        plan, done = eng.step_async()  # the host plans step k while the device runs step k - 1
        drv.advance(plan)
        return plan, done

    vis = os.environ.get("CUDA_VISIBLE_DEVICES", "")
    parts = vis.split(",") if vis else []
    phys = int(parts[local]) if len(parts) > local and parts[local].isdigit() else local
    sampler = ClockSampler(gpu_index=phys, period_ms=20).start()  # running before the window starts
    for _ in range(args.warmup):
        r = one_step()
        if r is None:
            break
        last_producers = [q.rid for q in ss.producers(r[0])]

    # 4. timed region (starts with nothing in flight). The set-up's objects
    # (2000 requests, the simulation's trace) move to a permanent generation,
    # so a cyclic garbage collection inside the window has little to walk: a
    # full collection over them once stalled the host for ~20 ms mid-window.
    eng.drain()
    gc.collect()
    gc.freeze()
    stream = torch.cuda.current_stream(dev)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    first_stat = len(eng.stats)
    launches0 = _ext.launches() + eng.graph_launches
    events = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps + 1)]
    produced = [last_producers]
    decode_tokens = prefill_tokens = 0
    finished = []
    d2h = 0
    wall0 = time.time()
    t_host0 = time.perf_counter()
    steps = 0
    host_ms = []
    for i in range(args.steps):
        events[i].record(stream)
        h0 = time.perf_counter()
        r = one_step()
        host_ms.append(1e3 * (time.perf_counter() - h0))
        if r is None:
            break
        plan, done = r
        decode_tokens += len(plan.decode)
        prefill_tokens += sum(n for _, _, n in plan.prefill)
        produced.append([q.rid for q in ss.producers(plan)])
        d2h += 4 * len(produced[-1])
        finished.extend(done)
        steps += 1
    events[steps].record(stream)
    finished.extend(eng.drain())  # the last step's tokens, read back to the host
    torch.cuda.synchronize(dev)
    t_host1 = time.perf_counter()
    wall1 = time.time()
    launches = _ext.launches() + eng.graph_launches - launches0
    if world > 1:
        dist.barrier()
    clocks = sampler.stop(window=(wall0, wall1))
    per_step = [events[i].elapsed_time(events[i + 1]) / 1e3 for i in range(steps)]
    dev_s = events[0].elapsed_time(events[steps]) / 1e3
    host_s = t_host1 - t_host0
    if world > 1:
        t = torch.tensor([dev_s, host_s] + per_step, dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        dev_s, host_s, per_step = float(t[0]), float(t[1]), t[2:].tolist()
    w = window_tpot(produced, per_step)
    fwd = [st.device_ms for st in eng.stats[first_stat:first_stat + steps]]
    # steps whose interval on the device exceeds their forward by over 1 ms:
    # [index, interval ms, forward ms, host ms of step_async, decode rows, prefill tokens]
    outliers = [[i, round(1e3 * per_step[i], 3), round(fwd[i], 3), round(host_ms[i], 3), eng.stats[first_stat + i].n_decode,
                 eng.stats[first_stat + i].n_prefill_tokens]
                for i in range(min(steps, len(fwd))) if 1e3 * per_step[i] - fwd[i] > 1.0]
    fin_tpot = sorted(x for x in (q.tpot() for q in finished) if x is not None)
    step_ms = [st.device_ms for st in eng.stats[first_stat:]]
    value = decode_tokens / dev_s if dev_s > 0 else 0.0
    e2e = decode_tokens / host_s if host_s > 0 else 0.0
    ms = lambda v: round(1e3 * v, 3) if v is not None else None  # noqa: E731
    out = {
        "metric": METRIC,
        "value": round(value, 2),
        "unit": "decode tokens/s",
        "n_gpus": world,
        "steps": steps,
        "warmup": args.warmup,
        "ms_per_step": round(1e3 * dev_s / max(steps, 1), 4),
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": (round(value / BASELINE_VALUE, 4) if BASELINE_VALUE else None),
        "dtype": "bf16",
        "data": "synthetic (random prompts, random-init weights; in-flight requests at the window start hold "
                "random KV)",
        "config": {
            "model": cfg.name + "-arch", "global_batch": f"continuous (max {args.max_batch})",
            "seq_len": args.prompt + args.output, "prompt_tokens": args.prompt,
            "output_tokens": args.output, "arrival": f"poisson {args.rate} req/s",
            "requests": args.requests, "parallelism": f"tp{world}",
            "tp_collective": (tp.mode if tp is not None else "none"),
            "levers": "pi+timer(1/8)+policy armed; acquire=" + args.acquire,
            "step_tokens": args.step_tokens or None,
            "l2": "inputs larger than L2 (16 GB of weights / N stream every step)",
            "window": dict(window, nominal_step_ms=round(step_s * 1e3, 3), nominal_prefill_us=round(tok_s * 1e6, 3),
                           workload_clock_s=round(drv.clock - window["t0_s"], 4)),
            "window_reproduced": (decode_tokens == window["window_decode_tokens"]
                                  and prefill_tokens == window["window_prefill_tokens"]),
            "mean_batch": round(decode_tokens / max(steps, 1), 3),
            "prefill_token_share": round(prefill_tokens / max(decode_tokens + prefill_tokens, 1), 4),
        },
        "p99_tpot_ms": ms(pct(w["tpot"], 99)),
        "p50_tpot_ms": ms(pct(w["tpot"], 50)),
        "p99_itl_ms": ms(pct(w["itl"], 99)),
        "p50_itl_ms": ms(pct(w["itl"], 50)),
        "tpot_requests": w["requests"],
        "finished_in_window": len(finished),
        "finished_p99_tpot_ms": ms(pct(fin_tpot, 99)),
        "step_ms_p50": round(float(np.median(step_ms)), 3) if step_ms else None,
        "step_ms_p99": round(pct(sorted(step_ms), 99), 3) if step_ms else None,
        # forward passes alone (per-step device times between the engine's
        # own events) against the whole window: the rest is host work between
        # forwards that the device waits for
        "forward_only_tok_s": (round(decode_tokens / (sum(step_ms) / 1e3), 2)
                               if step_ms and sum(step_ms) > 0 else None),
        "host_gap_share": (round(max(0.0, 1.0 - (sum(step_ms) / 1e3) / dev_s), 4)
                           if step_ms and dev_s > 0 else None),
        "gap_steps": outliers[:8],
        "e2e": {"value": round(e2e, 2), "unit": "decode tokens/s", "h2d_bytes_per_step": eng.packed_len * 4,
                "d2h_bytes_per_step": round(d2h / max(steps, 1), 1)},
        "gpu_launches": int(launches),
        "clocks": clocks,
        "impl": "ours",
    }
    if rank == 0:
        print(json.dumps(out))
    if world > 1:
        dist.barrier()
        eng.graphs.clear()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
