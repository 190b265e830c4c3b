"""Stand-in for the "reference NCCL build" on the serving workload: the
installed vLLM (its own FlashInfer/NCCL/cuBLAS stack, CUDA graphs) serving the
same Llama-3-8B-architecture decode workload as ``bench.py``.

The reference project itself cannot run here (no package metadata, and its
serving path needs clang+LLVM and SGLang, none of which are in the image), so
this is a clearly labelled stand-in, not the reference: an upstream serving
stack of the kind the reference plugs into, on the same box, same workload.

Workload (identical to ``bench.py``): Poisson arrivals at ``--rate`` req/s,
``--prompt`` random token ids, ``--output`` generated tokens (ignore_eos),
random-initialised bf16 weights (vLLM ``load_format="dummy"`` on a
Llama-3-8B config), greedy sampling. The engine is driven on the same
workload clock: each ``step()`` advances it by the step's wall time, and
arrivals up to the clock are admitted. Reported: decode tokens/s over the
timed steps and p50/p99 TPOT of the requests that finished in the window.

    python -m sched_pass_b200.benchmarks.vllm_standin --tp 1

``--steady-batch B`` instead times steady decode steps at a fixed batch: B
requests of ``--prompt`` tokens are prefilled, then ``--steps`` decode steps
are timed (host wall time per ``step()``, CUDA synchronised on both sides),
the shape ``benchmarks/decode_step.py`` times for this framework.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import tempfile
import time

import numpy as np

LLAMA3_8B = {
    "architectures": ["LlamaForCausalLM"], "model_type": "llama", "hidden_size": 4096,
    "intermediate_size": 14336, "num_hidden_layers": 32, "num_attention_heads": 32,
    "num_key_value_heads": 8, "head_dim": 128, "vocab_size": 128256, "rms_norm_eps": 1e-5,
    "rope_theta": 500000.0, "max_position_embeddings": 8192, "hidden_act": "silu",
    "tie_word_embeddings": False, "torch_dtype": "bfloat16", "bos_token_id": 128000,
    "eos_token_id": 128001,
}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--tp", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1500)
    ap.add_argument("--warmup", type=int, default=300)
    ap.add_argument("--rate", type=float, default=8.0)
    ap.add_argument("--prompt", type=int, default=1536)
    ap.add_argument("--output", type=int, default=128)
    ap.add_argument("--requests", type=int, default=2000)
    ap.add_argument("--max-batch", type=int, default=128)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--eager", action="store_true", help="no CUDA graphs / compilation")
    ap.add_argument("--steady-batch", type=int, default=0,
                    help="time decode steps of a fixed batch of this many requests instead")
    args = ap.parse_args()
    os.environ.setdefault("VLLM_ENABLE_V1_MULTIPROCESSING", "0")  # step() in this process

    from vllm import EngineArgs, LLMEngine, SamplingParams
    from vllm.inputs import TokensPrompt

    d = tempfile.mkdtemp(prefix="llama3_8b_cfg_")
    with open(os.path.join(d, "config.json"), "w") as f:
        json.dump(LLAMA3_8B, f)
    eng = LLMEngine.from_engine_args(EngineArgs(
        model=d, load_format="dummy", skip_tokenizer_init=True, dtype="bfloat16",
        tensor_parallel_size=args.tp, max_model_len=args.prompt + args.output + 64,
        max_num_seqs=args.max_batch, enforce_eager=args.eager, seed=args.seed,
        gpu_memory_utilization=0.85, disable_log_stats=True))

    if args.steady_batch:
        return steady(eng, args, SamplingParams, TokensPrompt)
    rng = np.random.default_rng(args.seed)
    arrivals = np.cumsum(rng.exponential(1.0 / args.rate, size=args.requests))
    prompts = rng.integers(0, LLAMA3_8B["vocab_size"], size=(args.requests, args.prompt))
    sp = SamplingParams(max_tokens=args.output, temperature=0.0, ignore_eos=True, detokenize=False)
    clock, nxt = 0.0, 0
    ntok: dict[str, int] = {}
    times: dict[str, list] = {}

    def admit():
        nonlocal nxt, clock
        while nxt < args.requests and arrivals[nxt] <= clock:
            rid = str(nxt)
            eng.add_request(rid, TokensPrompt(prompt_token_ids=prompts[nxt].tolist()), sp)
            ntok[rid], times[rid] = 0, []
            nxt += 1
        if not eng.has_unfinished_requests() and nxt < args.requests:
            clock = max(clock, float(arrivals[nxt]))
            admit()

    def step():
        nonlocal clock
        admit()
        if not eng.has_unfinished_requests():
            return None
        t0 = time.perf_counter()
        outs = eng.step()
        dt = time.perf_counter() - t0
        clock += dt
        new, done = 0, []
        for o in outs:
            n = len(o.outputs[0].token_ids)
            k = n - ntok[o.request_id]
            if k > 0:
                times[o.request_id] += [clock] * k
                ntok[o.request_id] = n
                new += k
            if o.finished:
                done.append(o.request_id)
        return dt, new, done

    for _ in range(args.warmup):
        if step() is None:
            break
    total_s, tokens, finished, steps = 0.0, 0, [], 0
    for _ in range(args.steps):
        r = step()
        if r is None:
            break
        dt, new, done = r
        total_s += dt
        tokens += new
        finished += done
        steps += 1
    tpots = sorted((times[r][-1] - times[r][0]) / (len(times[r]) - 1) for r in finished if len(times[r]) > 1)

    def pct(v, p):
        return float(v[min(len(v) - 1, int(math.ceil(p / 100.0 * len(v))) - 1)]) if v else None

    print(json.dumps({
        "impl": "vllm-standin", "vllm_tp": args.tp, "value": round(tokens / total_s, 2) if total_s else 0.0,
        "unit": "generated tokens/s (host step time)", "steps": steps, "warmup": args.warmup,
        "ms_per_step": round(1e3 * total_s / max(steps, 1), 4),
        "p50_tpot_ms": round(1e3 * pct(tpots, 50), 3) if tpots else None,
        "p99_tpot_ms": round(1e3 * pct(tpots, 99), 3) if tpots else None,
        "finished_in_window": len(finished), "cuda_graphs": not args.eager,
        "config": {"model": "llama-3-8b-arch (dummy weights)", "prompt_tokens": args.prompt,
                   "output_tokens": args.output, "arrival": f"poisson {args.rate} req/s"}}))


def steady(eng, args, SamplingParams, TokensPrompt):
    """Decode steps of a fixed batch (every request prefilled first)."""
    import torch
    rng = np.random.default_rng(args.seed)
    B = args.steady_batch
    sp = SamplingParams(max_tokens=args.steps + args.warmup + 64, temperature=0.0, ignore_eos=True,
                        detokenize=False)
    for i in range(B):
        eng.add_request(str(i), TokensPrompt(prompt_token_ids=rng.integers(0, LLAMA3_8B["vocab_size"],
                                                                           size=args.prompt).tolist()), sp)
    started = set()
    for _ in range(10 * B + 100):  # until every request has produced a token
        for o in eng.step():
            if o.outputs and len(o.outputs[0].token_ids) > 0:
                started.add(o.request_id)
        if len(started) == B:
            break
    for _ in range(args.warmup):
        eng.step()
    torch.cuda.synchronize()
    ts = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        eng.step()
        torch.cuda.synchronize()
        ts.append(time.perf_counter() - t0)
    med = float(np.median(ts))
    print(json.dumps({"impl": "vllm-standin", "mode": "steady-batch", "vllm_tp": args.tp, "batch": B,
                      "context": args.prompt, "step_ms_p50": round(1e3 * med, 4),
                      "step_ms_min": round(1e3 * min(ts), 4), "tok_s": round(B / med, 1), "steps": len(ts),
                      "cuda_graphs": not args.eager}))
    return 0


if __name__ == "__main__":
    main()
