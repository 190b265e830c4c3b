"""Steady-state window of an open-loop (Poisson) serving workload.

A window of K engine steps taken at the start of a run measures the start-up
transient: an empty engine, one or two requests in flight, no request old
enough to finish. This module finds a window of the same workload in steady
state and puts the engine's scheduler in the state it has at the window's
start without running the model for the steps before it:

1. ``simulate`` drives a fresh scheduler with the engine's configuration
   through the workload on a *nominal* clock: each step advances the clock by
   a fixed cost model of the step (a decode step's time plus a time per
   prefill token) and arrivals up to the clock are admitted. No model runs;
   sampled tokens are placeholders.
2. ``pick_window`` chooses, among the simulated steps after a warm-up
   horizon, the start s whose window [s + W, s + W + K) comes closest to the
   long-run means of both decode tokens per step and prefill tokens per step
   (a representative window; the choice is deterministic, so every rank and
   every GPU count picks the same s).
3. ``replay`` drives the engine's own scheduler through steps [0, s) the same
   way. The KV pages of the requests in flight then hold synthetic values,
   as their prompts and generated tokens are synthetic too.

Admissions in the warm-up and timed steps follow the same nominal clock, so
the window holds the same requests, batch sizes and prefill chunks at every
GPU count (a fixed load: strong scaling); only the device time differs.

The reference measures serving with SGLang's benchmark client against a live
server (jc-su/sched-pass scripts/bench_ab.sh:1-60); this window replaces the
live arrival clock so that a short device-timed run sees the same load as a
long one.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

# Nominal step cost on one B200 for the Llama-3-8B architecture (bf16): a
# decode-only step at the named workload's steady batch (4.29 ms median over a
# 1500-step run) and the added time per prefill token (a 1536-token prefill
# step takes about 33 ms).
NOMINAL_DECODE_STEP_S = 4.3e-3
NOMINAL_PREFILL_TOKEN_S = 19e-6


def nominal_cost(n_decode: int, n_prefill_tokens: int, decode_step_s: float = NOMINAL_DECODE_STEP_S,
                 prefill_token_s: float = NOMINAL_PREFILL_TOKEN_S) -> float:
    """Seconds the nominal clock advances for one step."""
    return decode_step_s + prefill_token_s * n_prefill_tokens


def producers(plan) -> list:
    """Requests that produce a token in a step: every decode request, and
    every prefill request whose chunk completes its prompt (the engine samples
    exactly these rows)."""
    out = list(plan.decode)
    out += [r for r, start, n in plan.prefill if start + n >= r.prompt_len]
    return out


def placeholder_token(req, vocab: int) -> int:
    """A deterministic token id for a simulated step (same on every rank)."""
    return int((req.rid * 7919 + req.total_len * 31) % max(vocab, 1))


@dataclass
class Trace:
    """Per simulated step: nominal clock at its start, decode tokens, prefill tokens."""
    clock: np.ndarray
    n_decode: np.ndarray
    n_prefill: np.ndarray


class Driver:
    """Steps a scheduler through a workload on the nominal clock."""

    def __init__(self, sched, reqs: list, vocab: int, cost=nominal_cost):
        self.sched = sched
        self.reqs = reqs
        self.vocab = vocab
        self.cost = cost
        self.clock = 0.0
        self.nxt = 0

    def admit(self, add=None) -> None:
        """Admit every arrival up to the clock; when nothing is left to run,
        jump the clock to the next arrival."""
        add = add or self.sched.add
        while self.nxt < len(self.reqs) and self.reqs[self.nxt].arrival <= self.clock:
            add(self.reqs[self.nxt])
            self.nxt += 1
        if self.sched.idle and self.nxt < len(self.reqs):
            self.clock = max(self.clock, self.reqs[self.nxt].arrival)
            self.admit(add)

    def advance(self, plan) -> None:
        self.clock += self.cost(len(plan.decode), sum(n for _, _, n in plan.prefill))

    def dry_step(self):
        """One step without a model: schedule, placeholder tokens, commit."""
        self.admit()
        if self.sched.idle:
            return None
        plan = self.sched.schedule()
        t0 = self.clock
        self.advance(plan)
        sampled = {r.rid: placeholder_token(r, self.vocab) for r in producers(plan)}
        self.sched.commit(plan, sampled, self.clock)
        return plan, t0


def clone_requests(reqs: list) -> list:
    """Fresh copies (same ids, prompts, arrivals, urgency) for a simulation."""
    from ..engine.request import Request
    return [Request(rid=r.rid, prompt=r.prompt, max_new_tokens=r.max_new_tokens, arrival=r.arrival,
                    urgency=r.urgency) for r in reqs]


def simulate(make_sched, reqs: list, vocab: int, until_s: float, cost=nominal_cost) -> Trace:
    """Simulate the workload on a fresh scheduler until the nominal clock
    passes ``until_s`` (or the workload ends)."""
    drv = Driver(make_sched(), clone_requests(reqs), vocab, cost)
    clock, nd, npf = [], [], []
    while drv.clock <= until_s:
        r = drv.dry_step()
        if r is None:
            break
        plan, t0 = r
        clock.append(t0)
        nd.append(len(plan.decode))
        npf.append(sum(n for _, _, n in plan.prefill))
    return Trace(np.asarray(clock), np.asarray(nd, dtype=np.int64), np.asarray(npf, dtype=np.int64))


def pick_window(trace: Trace, steps: int, warmup: int, horizon_s: float) -> tuple[int, dict]:
    """Start step s (the first warm-up step) of the most representative
    window: after ``horizon_s`` of workload, minimising the relative distance
    of the window's decode and prefill token totals from ``steps`` times
    their long-run means. Returns (s, summary)."""
    n = trace.clock.size
    first = int(np.searchsorted(trace.clock, horizon_s))
    last = n - (warmup + steps)
    if last < first:
        raise ValueError(f"workload too short: {n} simulated steps, need {first} + {warmup + steps}")
    nd = trace.n_decode[first:].astype(np.float64)
    npf = trace.n_prefill[first:].astype(np.float64)
    mu_d, mu_p = nd.mean(), npf.mean()
    cd = np.concatenate([[0.0], np.cumsum(trace.n_decode.astype(np.float64))])
    cp = np.concatenate([[0.0], np.cumsum(trace.n_prefill.astype(np.float64))])
    s = np.arange(first, last + 1)
    a, b = s + warmup, s + warmup + steps
    wd, wp = cd[b] - cd[a], cp[b] - cp[a]
    score = np.abs(wd - steps * mu_d) / max(steps * mu_d, 1e-9) + np.abs(wp - steps * mu_p) / max(steps * mu_p, 1.0)
    k = int(np.argmin(score))  # first minimum: deterministic
    best = int(s[k])
    return best, {"start_step": best, "t0_s": round(float(trace.clock[best]), 4),
                  "longrun_decode_per_step": round(float(mu_d), 3),
                  "longrun_prefill_tokens_per_step": round(float(mu_p), 2),
                  "window_decode_tokens": int(wd[k]), "window_prefill_tokens": int(wp[k]),
                  "score": round(float(score[k]), 4)}


def replay(sched, reqs: list, vocab: int, n_steps: int, cost=nominal_cost) -> Driver:
    """Drive ``sched`` (the engine's scheduler) through the first ``n_steps``
    steps of the workload without a model. Returns the driver, whose clock
    and next-arrival index continue the run."""
    drv = Driver(sched, reqs, vocab, cost)
    for _ in range(n_steps):
        if drv.dry_step() is None:
            break
    return drv
