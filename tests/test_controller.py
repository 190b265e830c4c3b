"""Closed-loop controller: estimator convergence, LPT, hysteresis (GPU-free)."""
import random

import numpy as np

from sched_pass_b200.runtime.controller import CostModel, SchedControlPlane


class FakePlane:
    def __init__(self):
        self.order, self.n, self.pushes = None, None, 0

    def set_order(self, o):
        self.order = list(o)

    def set_num_tasks(self, n):
        self.n = n

    def push(self):
        self.pushes += 1


def test_estimator_converges_and_lpt_matches_oracle():
    random.seed(0)
    ctl = SchedControlPlane(policy="lpt")
    plane = FakePlane()
    a_true, b_true = 7.5, 120.0
    rids = list(range(64))
    lens = [random.choice([64, 512]) for _ in rids]
    for _ in range(20):
        cyc = [a_true * ln + b_true + random.gauss(0, 5) for ln in lens]
        ctl.step(plane, rids, lens, cycles=cyc)
    a, _ = ctl.coeffs()
    assert abs(a - a_true) / a_true < 0.05
    got = ctl.order(rids, lens)
    assert [lens[i] for i in got] == sorted(lens, reverse=True)
    assert plane.pushes == 20 and plane.n == 64


def test_hysteresis_keeps_order_on_negligible_change():
    ctl = SchedControlPlane(policy="lpt")
    rids = list(range(16))
    lens = [100 * (i % 4 + 1) for i in rids]
    ctl.observe(rids, lens, [3.0 * x for x in lens])
    first = ctl.order(rids, lens)
    lens2 = list(lens)
    lens2[0] += 1
    assert ctl.order(rids, lens2) == first


def test_srpt_and_edf():
    ctl = SchedControlPlane(policy="srpt")
    ctl.observe([0, 1, 2], [10, 20, 30], [10, 20, 30])
    assert ctl.order([0, 1, 2], [30, 10, 20]) == [1, 2, 0]
    edf = SchedControlPlane(policy="edf")
    edf.observe([0, 1], [10, 20], [10, 20])
    assert edf.order([0, 1], [10, 10], deadlines=[100.0, 5.0]) == [1, 0]


def test_uncertainty_unobserved_is_full_doubt():
    ctl = SchedControlPlane()
    ctl.observe([0], [100], [100.0])
    assert ctl.uncertainty([5, 6], [100, 100]) == 1.0


def test_cost_model_degenerate_and_exact():
    f = CostModel()
    assert f.coeffs() == (1.0, 0.0)
    f.add([10], [30])
    assert f.coeffs() == (3.0, 0.0)
    f.add([10], [30])  # still one distinct x: proportional
    assert f.coeffs() == (3.0, 0.0)
    g = CostModel()
    g.add([1, 2, 3, 4], [5, 7, 9, 11])
    a, b = g.coeffs()
    assert abs(a - 2) < 1e-9 and abs(b - 3) < 1e-9


def test_batched_fit_equals_sample_by_sample_least_squares():
    rng = np.random.default_rng(1)
    x = rng.integers(16, 4096, size=300).astype(float)
    y = 3.5 * x + 800 + rng.normal(0, 40, size=x.size)
    batched, single = CostModel(), CostModel()
    for k in range(0, 300, 37):
        batched.add(x[k:k + 37], y[k:k + 37])
    for xi, yi in zip(x, y):
        single.add([xi], [yi])
    want = np.polyfit(x, y, 1)
    for m in (batched, single):
        assert np.allclose(m.coeffs(), want, rtol=1e-9)


def test_decay_follows_a_changed_cost():
    m = CostModel(decay=0.5)
    x = np.array([100.0, 200.0, 400.0])
    for _ in range(5):
        m.add(x, 2 * x)
    for _ in range(20):
        m.add(x, 5 * x)
    assert abs(m.coeffs()[0] - 5) < 1e-3


def test_residuals_are_per_request_and_forgotten():
    ctl = SchedControlPlane()
    lens = [100, 100, 200, 200]
    for _ in range(40):
        # request 7 always runs 50 % slower than its length says
        ctl.observe([5, 7, 8, 9], lens, [10.0 * l * (1.5 if r == 7 else 1.0) for r, l in zip([5, 7, 8, 9], lens)])
    assert ctl.predict_one(100, rid=7) > 1.3 * ctl.predict_one(100, rid=5)
    order = ctl.order([5, 7, 8, 9], lens)
    assert order[:2] in ([2, 3], [3, 2]) and order[2] == 1  # the slow short request before its peer
    ctl.forget([7])
    assert ctl.predict_one(100, rid=7) == ctl.predict_one(100)
    assert ctl.uncertainty([7], [100]) == 1.0  # unknown again: full doubt


def test_families_are_separate():
    ctl = SchedControlPlane()
    ctl.observe([1, 2], [100, 200], [100.0, 200.0], family="decode")
    ctl.observe([1, 2], [100, 200], [1000.0, 2000.0], family="prefill")
    assert abs(ctl.predict_one(300) - 300) < 1e-6
    assert abs(ctl.predict_one(300, family="prefill") - 3000) < 1e-6
