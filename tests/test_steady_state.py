"""Steady-state window of the bench (CPU): the simulated scheduler picks a
representative window, a replay on a second scheduler reproduces the
simulated steps exactly, and the window's inter-token statistics only use
intervals that lie inside the window."""
import os
import sys

import numpy as np

from sched_pass_b200.benchmarks import steady_state as ss
from sched_pass_b200.engine.request import Request
from sched_pass_b200.engine.scheduler import Scheduler

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)
import bench  # noqa: E402

VOCAB = 1000


def workload(n=400, rate=8.0, prompt=1536, out=128, seed=0):
    rng = np.random.default_rng(seed)
    arr = np.cumsum(rng.exponential(1.0 / rate, size=n))
    P = rng.integers(0, VOCAB, size=(n, prompt)).astype(np.int32)
    return [Request(rid=i, prompt=P[i], max_new_tokens=out, arrival=float(arr[i])) for i in range(n)]


def make():
    return Scheduler(128 * 112 + 64, 16, 128, 2048, 1792)


def test_window_is_representative_and_deterministic():
    reqs = workload()
    tr = ss.simulate(make, reqs, VOCAB, 40.0)
    s, win = ss.pick_window(tr, 20, 5, 15.0)
    s2, win2 = ss.pick_window(ss.simulate(make, reqs, VOCAB, 40.0), 20, 5, 15.0)
    assert (s, win) == (s2, win2)
    assert tr.clock[s] >= 15.0
    # the long-run batch of 8 req/s x ~0.7 s request lifetime is about 5-6
    assert 4.0 < win["longrun_decode_per_step"] < 8.0
    assert abs(win["window_decode_tokens"] - 20 * win["longrun_decode_per_step"]) < 0.25 * 20 * win[
        "longrun_decode_per_step"]
    assert win["window_prefill_tokens"] > 0  # the window holds arrivals, as the long run does


def test_replay_reproduces_the_simulated_steps():
    reqs = workload()
    tr = ss.simulate(make, reqs, VOCAB, 40.0)
    s, _ = ss.pick_window(tr, 20, 5, 15.0)
    fresh = ss.clone_requests(reqs)
    sched = make()
    drv = ss.replay(sched, fresh, VOCAB, s)
    assert abs(drv.clock - tr.clock[s]) < 1e-9
    for k in range(25):  # the warm-up and timed steps continue the same way
        r = drv.dry_step()
        assert r is not None
        plan, t0 = r
        assert abs(t0 - tr.clock[s + k]) < 1e-9
        assert len(plan.decode) == tr.n_decode[s + k]
        assert sum(n for _, _, n in plan.prefill) == tr.n_prefill[s + k]


def test_window_tpot_counts_only_intervals_inside_the_window():
    # request 1 decodes every step; request 2 arrives at step 1 (first token
    # from its prefill, no interval) and decodes at steps 2 and 3
    produced = [[1], [1], [1, 2], [1, 2], [1, 2]]
    step_s = [0.01, 0.03, 0.01, 0.01]
    w = bench.window_tpot(produced, step_s)
    assert w["requests"] == 2
    assert np.allclose(sorted(w["itl"]), sorted([0.01, 0.03, 0.01, 0.01, 0.01, 0.01]))
    assert np.allclose(w["tpot"], sorted([np.mean([0.01, 0.03, 0.01, 0.01]), 0.01]))
    assert np.isclose(bench.pct(w["itl"], 99), 0.03) and np.isclose(bench.pct(w["itl"], 50), 0.01)
