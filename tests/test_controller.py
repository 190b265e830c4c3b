"""Closed-loop controller: estimator convergence, LPT, hysteresis (GPU-free)."""
import random

from sched_pass_b200.runtime.controller import LineFit, SchedControlPlane


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
    a, _ = ctl._fit.coeffs()
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


def test_linefit_degenerate():
    f = LineFit()
    assert f.coeffs() == (1.0, 0.0)
    f.add(10, 30)
    assert f.coeffs() == (3.0, 0.0)
