"""Serving A/B of the scheduling plane: the same workload through the engine
with the levers off ("stock"), learning costs without installing anything
("observe"), and installing orders / CLC / hints ("enforce"); optionally
"enforce-noclc" (acquisition pinned to static + pi). The reference runs the
same three arms against SGLang (scripts/bench_ab.sh:56-58) and warns that
end-to-end serving numbers swing 10-25 % between identical runs
(jc-su/sched-pass ROADMAP.md:854-857), so the arms are interleaved over ``--repeats`` rounds
on one set of weights and the summary keeps the best round per arm.

    python -m sched_pass_b200.benchmarks.serving_ab --mix dispersed --requests 400 --repeats 3

One JSON line per (round, arm) and a final ``{"summary": ...}`` line with
TPOT p50/p99, TTFT p50, and output tokens per second of the workload clock
(device step time plus idle gaps).
"""
from __future__ import annotations

import argparse
import json
import os

ARMS = {
    "stock": ({"levers": False}, {}),
    "observe": ({"levers": True, "acquire": "auto"}, {"SCHED_ENFORCE": "0"}),
    "enforce": ({"levers": True, "acquire": "auto"}, {"SCHED_ENFORCE": "1"}),
    "enforce-noclc": ({"levers": True, "acquire": "static"}, {"SCHED_ENFORCE": "1", "SCHED_CLC_ARM": "off"}),
}


def run_ab(make_engine, work, arms, repeats: int, emit=print) -> dict:
    """``make_engine(engine_kwargs)`` builds a fresh engine for one arm (the
    arm's SCHED_* variables are set while it is built and run). Returns the
    best round per arm (lowest TPOT p50)."""
    from ..engine import loadgen
    best = {}
    for rnd in range(repeats):
        for arm in arms:
            kw, env = ARMS[arm]
            saved = {k: os.environ.get(k) for k in env}
            os.environ.update(env)
            try:
                eng = make_engine(dict(kw))
                res, wall = loadgen.run_inprocess(eng, work)
            finally:
                for k, v in saved.items():
                    if v is None:
                        os.environ.pop(k, None)
                    else:
                        os.environ[k] = v
            s = loadgen.summarize(res, wall, tag=arm)
            rec = {"round": rnd, "arm": arm, "n_ok": s["n_ok"], "out_tok_per_s": s["out_tok_per_s"],
                   "tpot_p50_ms": _ms(s["tpot_p50"]), "tpot_p99_ms": _ms(s["tpot_p99"]),
                   "ttft_p50_ms": _ms(s["ttft_p50"])}
            emit(json.dumps(rec))
            if arm not in best or (rec["tpot_p50_ms"] or 1e30) < (best[arm]["tpot_p50_ms"] or 1e30):
                best[arm] = rec
            del eng
    emit(json.dumps({"summary": best}))
    return best


def _ms(v):
    return None if v is None else round(1e3 * v, 3)


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="llama-3-8b")
    ap.add_argument("--arms", default="stock,observe,enforce")
    ap.add_argument("--mix", default="poisson", choices=["poisson", "dispersed"])
    ap.add_argument("--requests", type=int, default=400)
    ap.add_argument("--rate", type=float, default=8.0)
    ap.add_argument("--prompt", type=int, default=1536)
    ap.add_argument("--output", type=int, default=128)
    ap.add_argument("--max-batch", type=int, default=128)
    ap.add_argument("--repeats", type=int, default=3)
    ap.add_argument("--seed", type=int, default=0)
    a = ap.parse_args(argv)
    import torch

    from ..engine import loadgen
    from ..engine.engine import Engine, EngineConfig
    from ..models.config import get_config
    from ..models.llama import init_weights

    cfg = get_config(a.model)
    dev = torch.device("cuda", torch.cuda.current_device())
    weights = init_weights(cfg, dev, seed=a.seed)
    if a.mix == "poisson":
        work = loadgen.poisson(a.requests, a.rate, a.prompt, a.output, vocab=cfg.vocab, seed=a.seed)
    else:
        work = loadgen.dispersed(a.requests, hi=a.prompt, out=a.output, vocab=cfg.vocab, seed=a.seed, rate=a.rate)
    max_ctx = (max(len(w.prompt) for w in work) + a.output + 16 + 127) // 128 * 128

    def make_engine(kw):
        torch.cuda.empty_cache()
        ecfg = EngineConfig(max_batch=a.max_batch, max_prefill_tokens=2048, max_context=max_ctx, seed=a.seed, **kw)
        return Engine(cfg, ecfg, dev, weights=weights)

    run_ab(make_engine, work, a.arms.split(","), a.repeats)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
