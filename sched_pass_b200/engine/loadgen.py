"""Load generation for the serving engine: trace replay and synthetic mixes.

Trace replay (the reference's python/sched_trace_loadgen.py:36-142 contract):
a Qwen-Bailian-style trace is a JSONL of records with ``timestamp``,
``input_length``, ``output_length`` and ``hash_ids`` (one id per 16-token KV
block). Every hash id maps to a fixed block of 16 token ids
(``block_tokens``), and a request's prompt is the concatenation of its
blocks cut to ``input_length`` (``craft_prompt``) -- so two records that
share a prefix of hash ids share the same prefix of tokens, and the trace's
prefix reuse survives the reconstruction exactly.

Synthetic mixes: ``dispersed`` (log-normal prompt lengths with a fixed
seed: the reference's test/py/loadgen_dispersed.py:23-37 straggler mix) and
``poisson`` (fixed-length prompts with Poisson arrivals: the serving
benchmark's workload).

Drivers: ``run_inprocess`` feeds an ``Engine`` on its workload clock (arrivals
admitted as the clock passes them) and ``replay_http`` posts to any
``/generate`` endpoint (this package's server or another one) with bounded
concurrency. ``summarize`` reports p50/p90/p99 of latency, TTFT and TPOT.

    python -m sched_pass_b200.engine.loadgen --selftest
    python -m sched_pass_b200.engine.loadgen --trace t.jsonl --base-url http://127.0.0.1:30000
"""
from __future__ import annotations

import argparse
import functools
import json
import math
import os
import sys
import time
from dataclasses import dataclass, field

import numpy as np

BLOCK = 16


@functools.lru_cache(maxsize=1 << 16)
def _block(hash_id: int, vocab: int, block: int) -> tuple:
    # a counter-based generator keyed by the hash id: the same id gives the
    # same block in every process, and nearby ids give unrelated blocks
    g = np.random.Generator(np.random.Philox(key=[int(hash_id) & 0xFFFFFFFFFFFFFFFF, 0x51ED5C4ED]))
    return tuple(int(t) for t in g.integers(0, vocab, size=block))


def block_tokens(hash_id: int, vocab: int = 128256, block: int = BLOCK) -> list:
    """The fixed ``block`` token ids of one KV-block hash id."""
    return list(_block(int(hash_id), int(vocab), int(block)))


def craft_prompt(rec: dict, vocab: int = 128256, block: int = BLOCK) -> np.ndarray:
    """Prompt token ids of a trace record: its blocks, cut (or padded with a
    per-record block) to ``input_length``."""
    want = int(rec.get("input_length", 0)) or block
    out: list = []
    for h in rec.get("hash_ids", []):
        out.extend(_block(int(h), vocab, block))
        if len(out) >= want:
            break
    if len(out) < want:
        pad = _block((1 << 62) + int(rec.get("chat_id", 0)), vocab, block)
        while len(out) < want:
            out.extend(pad)
    return np.asarray(out[:want], dtype=np.int32)


def load_trace(path: str, limit: int | None = None) -> list:
    """Records sorted by timestamp; a truncated last line (a partial
    download) ends the read instead of failing it."""
    recs = []
    with open(path) as f:
        for line in f:
            line = line.strip()
            if not line:
                continue
            try:
                recs.append(json.loads(line))
            except json.JSONDecodeError:
                break
            if limit and len(recs) >= limit:
                break
    recs.sort(key=lambda r: float(r.get("timestamp", 0.0)))
    return recs


@dataclass
class WorkItem:
    prompt: np.ndarray
    max_new_tokens: int
    arrival: float = 0.0       # seconds from the start of the run
    urgency: float = 0.0
    tag: str = ""


def from_trace(recs: list, vocab: int, speed: float = 1.0, max_output: int | None = None) -> list:
    t0 = float(recs[0].get("timestamp", 0.0)) if recs else 0.0
    out = []
    for r in recs:
        n_out = max(1, int(r.get("output_length", 1)))
        if max_output:
            n_out = min(n_out, max_output)
        arr = (float(r.get("timestamp", 0.0)) - t0) / speed if speed > 0 else 0.0
        out.append(WorkItem(craft_prompt(r, vocab), n_out, arr, tag=str(r.get("type", ""))))
    return out


def dispersed(n: int, mu: float = 5.8, sigma: float = 1.1, lo: int = 32, hi: int = 1536, out: int = 128,
              vocab: int = 128256, seed: int = 42, rate: float = 0.0) -> list:
    """Log-normal prompt lengths exp(N(mu, sigma)) clipped to [lo, hi], fixed
    output length; all at t=0 (closed loop) unless ``rate`` > 0 (Poisson)."""
    rng = np.random.default_rng(seed)
    lens = np.clip(np.rint(np.exp(rng.normal(mu, sigma, size=n))), lo, hi).astype(np.int64)
    arr = np.cumsum(rng.exponential(1.0 / rate, size=n)) if rate > 0 else np.zeros(n)
    return [WorkItem(rng.integers(0, vocab, size=int(L)).astype(np.int32), out, float(a),
                     urgency=float(rng.random())) for L, a in zip(lens, arr)]


def poisson(n: int, rate: float, prompt: int, out: int, vocab: int = 128256, seed: int = 0) -> list:
    rng = np.random.default_rng(seed)
    arr = np.cumsum(rng.exponential(1.0 / rate, size=n))
    return [WorkItem(rng.integers(0, vocab, size=prompt).astype(np.int32), out, float(a),
                     urgency=float(rng.random())) for a in arr]


@dataclass
class Result:
    ok: bool
    latency: float
    ttft: float | None = None
    tpot: float | None = None
    n_in: int = 0
    n_out: int = 0
    extra: dict = field(default_factory=dict)


def run_inprocess(engine, work: list, max_steps: int | None = None) -> tuple[list, float]:
    """Drive ``engine`` on its workload clock: a request is admitted once the
    clock passes its arrival; when idle, the clock jumps to the next arrival.
    Returns (results, workload seconds)."""
    from .request import Request
    reqs = [Request(rid=i, prompt=w.prompt, max_new_tokens=w.max_new_tokens, arrival=w.arrival,
                    urgency=w.urgency) for i, w in enumerate(work)]
    order = sorted(range(len(reqs)), key=lambda i: reqs[i].arrival)
    nxt, steps = 0, 0
    clock0 = engine.clock
    for r in reqs:
        r.arrival += clock0
    while True:
        while nxt < len(order) and reqs[order[nxt]].arrival <= engine.clock:
            engine.add_request(reqs[order[nxt]])
            nxt += 1
        if not engine.has_work():
            if nxt >= len(order):
                break
            engine.clock = max(engine.clock, reqs[order[nxt]].arrival)
            continue
        engine.step()
        steps += 1
        if max_steps is not None and steps >= max_steps:
            break
    res = []
    for r in reqs:
        done = r.finished and r.token_times
        res.append(Result(ok=bool(done), latency=(r.token_times[-1] - r.arrival) if done else float("nan"),
                          ttft=r.ttft(), tpot=r.tpot(), n_in=r.prompt_len, n_out=len(r.output)))
    return res, engine.clock - clock0


async def _post(session, url, w: WorkItem, sem, results, idx, stream: bool = False):
    payload = {"input_ids": [int(t) for t in w.prompt],
               "sampling_params": {"max_new_tokens": w.max_new_tokens, "temperature": 0.0, "ignore_eos": True}}
    if stream:
        return await _post_stream(session, url, w, sem, results, idx, payload)
    async with sem:
        t0 = time.perf_counter()
        try:
            async with session.post(url, json=payload) as r:
                body = await r.json()
                ok = r.status == 200
        except Exception as e:  # noqa: BLE001 - a failed request is a result
            body, ok = {"error": repr(e)}, False
        dt = time.perf_counter() - t0
    meta = body.get("meta_info", {}) if isinstance(body, dict) else {}
    results[idx] = Result(ok=ok, latency=dt, ttft=meta.get("ttft"), tpot=meta.get("tpot"),
                          n_in=len(w.prompt), n_out=len(body.get("output_ids", [])) if ok else 0)


async def _post_stream(session, url, w: WorkItem, sem, results, idx, payload):
    """Streaming request: TTFT and TPOT measured on the client's clock from
    the arrival times of the server-sent token events (what a user sees),
    instead of the server's own accounting."""
    payload = dict(payload, stream=True)
    times, n, ok = [], 0, False
    async with sem:
        t0 = time.perf_counter()
        try:
            async with session.post(url, json=payload) as r:
                async for raw in r.content:
                    line = raw.decode().strip()
                    if not line.startswith("data: "):
                        continue
                    ev = json.loads(line[len("data: "):])
                    if ev.get("done"):
                        ok = r.status == 200 and "error" not in ev
                        break
                    times.append(time.perf_counter())
                    n += 1
        except Exception:  # noqa: BLE001 - a failed request is a result
            ok = False
        dt = time.perf_counter() - t0
    ttft = times[0] - t0 if times else None
    tpot = (times[-1] - times[0]) / (len(times) - 1) if len(times) > 1 else None
    results[idx] = Result(ok=ok, latency=dt, ttft=ttft, tpot=tpot, n_in=len(w.prompt), n_out=n,
                          extra={"client_clock": True})


async def replay_http_async(base_url: str, work: list, concurrency: int = 32, realtime: bool = True,
                            stream: bool = False) -> list:
    import asyncio

    import aiohttp
    sem = asyncio.Semaphore(concurrency)
    results: list = [None] * len(work)
    url = base_url.rstrip("/") + "/generate"
    t_start = time.perf_counter()
    timeout = aiohttp.ClientTimeout(total=3600)
    async with aiohttp.ClientSession(timeout=timeout,
                                     connector=aiohttp.TCPConnector(limit=concurrency + 8)) as s:
        tasks = []
        for i in sorted(range(len(work)), key=lambda k: work[k].arrival):
            if realtime:
                due = work[i].arrival - (time.perf_counter() - t_start)
                if due > 0:
                    await asyncio.sleep(due)
            tasks.append(asyncio.create_task(_post(s, url, work[i], sem, results, i, stream)))
        await asyncio.gather(*tasks)
    return results


def replay_http(base_url: str, work: list, concurrency: int = 32, realtime: bool = True,
                stream: bool = False) -> tuple[list, float]:
    """Replay ``work`` against ``/generate``. ``stream``: request server-sent
    token events and measure TTFT / TPOT on the client's clock."""
    import asyncio
    t0 = time.perf_counter()
    res = asyncio.run(replay_http_async(base_url, work, concurrency, realtime, stream))
    return res, time.perf_counter() - t0


def _pct(v: list, p: float):
    if not v:
        return None
    v = sorted(v)
    return float(v[min(len(v) - 1, max(0, int(math.ceil(p * len(v))) - 1))])


def summarize(results: list, wall_s: float, tag: str = "", stream=None) -> dict:
    ok = [r for r in results if r is not None and r.ok]
    lat = [r.latency for r in ok]
    ttft = [r.ttft for r in ok if r.ttft is not None]
    tpot = [r.tpot for r in ok if r.tpot is not None]
    out_tok = sum(r.n_out for r in ok)
    s = {"tag": tag, "n": len(results), "n_ok": len(ok), "wall_s": wall_s,
         "req_per_s": len(ok) / wall_s if wall_s > 0 else None,
         "out_tok_per_s": out_tok / wall_s if wall_s > 0 else None}
    for name, v in (("latency", lat), ("ttft", ttft), ("tpot", tpot)):
        for p in (0.5, 0.9, 0.99):
            s[f"{name}_p{int(p * 100)}"] = _pct(v, p)
    if stream is not None:
        print(f"== load summary {tag} ==", file=stream)
        print(f"  requests : {s['n_ok']}/{s['n']} ok in {wall_s:.2f}s "
              f"({(s['req_per_s'] or 0):.2f} req/s, {(s['out_tok_per_s'] or 0):.1f} tok/s)", file=stream)
        for name in ("latency", "ttft", "tpot"):
            vals = [s[f"{name}_p{q}"] for q in (50, 90, 99)]
            if vals[0] is not None:
                print(f"  {name:8s} : p50={vals[0]:.4f} p90={vals[1]:.4f} p99={vals[2]:.4f} s", file=stream)
    return s


def selftest(trace: str | None = None) -> int:
    """Offline checks of the reconstruction (no engine, no server)."""
    fails = 0

    def check(c, what):
        nonlocal fails
        print(f"  [{'PASS' if c else 'FAIL'}] {what}")
        fails += 0 if c else 1

    check(block_tokens(7) == block_tokens(7), "block of a hash id is fixed")
    check(block_tokens(7) != block_tokens(8), "different hash ids give different blocks")
    a = craft_prompt({"chat_id": 1, "input_length": 96, "hash_ids": [10, 11, 12, 13, 14, 15]})
    b = craft_prompt({"chat_id": 2, "input_length": 96, "hash_ids": [10, 11, 12, 90, 91, 92]})
    check(len(a) == len(b) == 96, "prompt length == input_length")
    check(np.array_equal(a[:48], b[:48]) and not np.array_equal(a[48:], b[48:]),
          "shared 3-block prefix -> shared 48-token prefix, divergent tail")
    check(len(craft_prompt({"input_length": 40, "hash_ids": [1, 2, 3, 4]})) == 40, "cut inside a block")
    check(len(craft_prompt({"chat_id": 5, "input_length": 200, "hash_ids": [1, 2]})) == 200,
          "padded when the hash ids run out")
    d = dispersed(2000, seed=3)
    lens = np.array([len(w.prompt) for w in d])
    check(lens.min() >= 32 and lens.max() <= 1536 and np.percentile(lens, 99) / np.median(lens) > 4,
          "dispersed mix is heavy-tailed within bounds")
    check([len(w.prompt) for w in dispersed(50, seed=3)] == [len(w.prompt) for w in dispersed(50, seed=3)],
          "dispersed mix is reproducible")
    if trace and os.path.exists(trace):
        recs = load_trace(trace)
        check(len(recs) > 0, f"trace parsed ({len(recs)} records)")
        check(all(len(craft_prompt(r)) == int(r["input_length"]) for r in recs), "every prompt length exact")
        seen, tot, rep = set(), 0, 0
        for r in recs:
            for h in r.get("hash_ids", []):
                tot += 1
                rep += h in seen
                seen.add(h)
        seen_b, tb, rb = set(), 0, 0
        for r in recs:
            p = craft_prompt(r)
            for i in range(0, len(p) // BLOCK * BLOCK, BLOCK):
                k = p[i:i + BLOCK].tobytes()
                tb += 1
                rb += k in seen_b
                seen_b.add(k)
        check(abs(rep / max(tot, 1) - rb / max(tb, 1)) < 0.01, "block reuse of prompts == hash reuse of trace")
    print("== ALL PASS ==" if not fails else f"== {fails} FAILED ==")
    return fails


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--selftest", action="store_true")
    ap.add_argument("--trace")
    ap.add_argument("--limit", type=int)
    ap.add_argument("--speed", type=float, default=1.0, help="trace time compression (0: all at once)")
    ap.add_argument("--base-url", help="a /generate endpoint; without it the engine runs in-process")
    ap.add_argument("--concurrency", type=int, default=32)
    ap.add_argument("--stream", action="store_true", help="stream tokens; TTFT/TPOT on the client's clock")
    ap.add_argument("--prefix-cache", action="store_true", help="in-process engine: share prompt-prefix KV pages")
    ap.add_argument("--admission", default="fcfs", choices=["fcfs", "urgency", "lpm"])
    ap.add_argument("--mix", default="trace", choices=["trace", "dispersed", "poisson"])
    ap.add_argument("--n", type=int, default=256)
    ap.add_argument("--rate", type=float, default=8.0)
    ap.add_argument("--prompt", type=int, default=1536)
    ap.add_argument("--output", type=int, default=128)
    ap.add_argument("--model", default="llama-3-8b")
    ap.add_argument("--vocab", type=int, default=None)
    a = ap.parse_args(argv)
    if a.selftest:
        return selftest(a.trace)
    from ..models.config import get_config
    cfg = get_config(a.model)
    vocab = a.vocab or cfg.vocab
    if a.mix == "trace":
        if not a.trace:
            print("--trace is required for --mix trace", file=sys.stderr)
            return 2
        work = from_trace(load_trace(a.trace, a.limit), vocab, a.speed, max_output=a.output)
    elif a.mix == "dispersed":
        work = dispersed(a.n, out=a.output, vocab=vocab, rate=a.rate)
    else:
        work = poisson(a.n, a.rate, a.prompt, a.output, vocab)
    if a.base_url:
        res, wall = replay_http(a.base_url, work, a.concurrency, stream=a.stream)
    else:
        import torch

        from .engine import Engine, EngineConfig
        longest = max(len(w.prompt) + w.max_new_tokens for w in work)
        eng = Engine(cfg, EngineConfig(max_batch=128, max_context=(longest + 127) // 128 * 128,
                                       prefix_cache=a.prefix_cache, admission=a.admission),
                     torch.device("cuda"))
        res, wall = run_inprocess(eng, work)
        if eng.sched.cache is not None:
            c = eng.sched.cache
            print(f"  prefix cache: {c.hits}/{c.lookups} prompt tokens served from cached pages")
    summarize(res, wall, a.mix, stream=sys.stdout)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
