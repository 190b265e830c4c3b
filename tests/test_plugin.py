"""Scheduling plugin on the CPU: typed config <-> SCHED_* env, regime gates,
failure isolation of hooks (a fake engine and plane stand in for the GPU)."""
import io

import numpy as np
import torch

from sched_pass_b200.engine.plugin import HookRunner, SchedPlugin, SchedPluginConfig
from sched_pass_b200.runtime.controller import SchedControlPlane


class FakePlane:
    def __init__(self, n=4096):
        self.N = n
        self.log = []
        self.timer_t = torch.zeros(n, dtype=torch.int64)

    def install_order(self, order, n):
        self.log.append(("order", int(n), order.clone()))

    def set_order_size(self, n):
        self.log.append(("order_size", n))

    def reset_order(self):
        self.log.append(("reset",))

    def set_num_tasks(self, n):
        self.log.append(("num_tasks", n))

    def set_timer_enabled(self, on):
        self.log.append(("timer", bool(on)))

    def clear_timer(self):
        self.timer_t.zero_()

    def set_rows(self, q=None, tau=None, hint=None, n=None):
        self.log.append(("rows", None if q is None else q.copy(), None if tau is None else tau.copy(), n))

    def push(self):
        self.log.append(("push",))


class Req:
    def __init__(self, rid, n, urgency):
        self.rid, self.total_len, self.urgency, self.tau = rid, n, urgency, 0


class Plan:
    def __init__(self, dec):
        self.decode = dec


class Ecfg:
    levers = True
    acquire = "auto"


class FakeEngine:
    def __init__(self, lens, R=8, hkv=2):
        self.R, self.hkv, self.step_no = R, hkv, 0
        self.plane = FakePlane()
        self.controller = SchedControlPlane(policy="lpt")
        self.ecfg = Ecfg()
        self.hooks = HookRunner(stream=io.StringIO())
        self.items = np.zeros((len(lens), 4), dtype=np.int32)
        for i, n in enumerate(lens):
            self.items[i] = (i, 0, n, 0)  # one item per request: (req, first page, tokens, split)
        self.plan = Plan([Req(i, n, u) for i, (n, u) in enumerate(zip(lens, np.linspace(0, 1, len(lens))))])

    def _host(self, name):
        assert name == "items"
        return self.items.reshape(-1)

    def info(self):
        return {"nd": len(self.plan.decode), "n_items": len(self.items), "S": 1}


def test_config_env_roundtrip_and_validation():
    c = SchedPluginConfig(timer_every=3, clc="on", shed_fraction=0.25, enforce=False)
    env = c.to_env()
    assert env["SCHED_TIMER_EVERY"] == "3" and env["SCHED_CLC_ARM"] == "on" and env["SCHED_ENFORCE"] == "0"
    back = SchedPluginConfig.from_env(env)
    assert back == c
    try:
        SchedPluginConfig.from_env({"SCHED_CLC_ARM": "maybe"})
    except ValueError:
        pass
    else:
        raise AssertionError("bad knob value accepted")


def test_one_wave_retires_order_and_queued_installs_lpt():
    eng = FakeEngine([100, 200, 50], R=64)  # 6 tasks <= R: one wave
    p = SchedPlugin(SchedPluginConfig(timer_every=0, clc="off"))
    p.on_batch_begin(eng, eng.plan, eng.info())
    kinds = [e[0] for e in eng.plane.log]
    assert "order" not in kinds and ("order_size", 0) in eng.plane.log and kinds[-1] == "push"
    lens = list(np.random.default_rng(0).integers(16, 4000, size=40))
    eng = FakeEngine(lens, R=8)  # 80 tasks > R: queued
    p.on_batch_begin(eng, eng.plan, eng.info())
    orders = [e for e in eng.plane.log if e[0] == "order"]
    assert len(orders) == 1 and orders[0][1] == 80
    assert sorted(orders[0][2].tolist()) == list(range(80))  # a permutation
    assert p.stats.orders["lpt"] == 1


def test_clc_arms_only_on_imbalance_and_uncertainty():
    lens = [4000] * 2 + [20] * 60  # one-sided tail: max/mean large
    eng = FakeEngine(lens, R=8)
    p = SchedPlugin(SchedPluginConfig(timer_every=0, clc="auto", clc_imbalance=3.0, clc_resid=0.5))
    p.on_batch_begin(eng, eng.plan, eng.info())  # cold estimator: uncertainty 1.0
    assert p.stats.clc_armed == 1 and p.stats.orders["region"] == 1
    uniform = FakeEngine([500] * 62, R=8)
    p2 = SchedPlugin(SchedPluginConfig(timer_every=0, clc="auto", clc_imbalance=3.0, clc_resid=0.5))
    p2.on_batch_begin(uniform, uniform.plan, uniform.info())
    assert p2.stats.clc_armed == 0 and p2.stats.orders["lpt"] == 1


def test_observe_mode_installs_nothing_and_probes_fold():
    eng = FakeEngine([300, 30, 3000, 40] * 10, R=8)
    p = SchedPlugin(SchedPluginConfig(timer_every=1, enforce=False))
    p.on_batch_begin(eng, eng.plan, eng.info())
    assert not any(e[0] in ("order", "num_tasks") for e in eng.plane.log)
    assert ("timer", True) in eng.plane.log
    # pretend the kernel timed every task: cost proportional to length
    lens = np.array([r.total_len for r in eng.plan.decode])
    eng.plane.timer_t[: len(lens) * eng.hkv] = torch.from_numpy(np.repeat(lens * 10, eng.hkv))
    p.on_batch_end(eng, eng.plan, eng.info(), 1.0)
    assert p.stats.probes == 1
    # the fit learned ~10 cycles per token (2 heads of 10 per token each)
    assert abs(eng.controller.predict_one(1000) / 1000 - 20) < 2


def test_shed_sets_tau_on_lowest_urgency():
    eng = FakeEngine([400, 800, 1200, 1600], R=64)
    p = SchedPlugin(SchedPluginConfig(timer_every=0, shed_fraction=0.5, shed_ratio=0.5))
    p.on_batch_begin(eng, eng.plan, eng.info())
    rows = [e for e in eng.plane.log if e[0] == "rows" and e[2] is not None][-1]
    tau = rows[2].reshape(-1, eng.hkv)[:, 0]
    assert list(tau) == [200, 400, 0, 0]  # urgencies rise with the index


def test_hook_errors_are_isolated_and_logged_once():
    class Bad:
        def on_batch_begin(self, *a):
            raise RuntimeError("boom")

        def on_batch_end(self, *a):
            raise KeyError("x")

    out = io.StringIO()
    h = HookRunner(stream=out)
    h.register(Bad())
    good = SchedPlugin(SchedPluginConfig(timer_every=0))
    h.register(good)
    eng = FakeEngine([10, 20], R=64)
    eng.hooks = h
    for _ in range(3):
        h.begin(eng, eng.plan, eng.info())
        h.end(eng, eng.plan, eng.info(), 0.1)
    assert h.errors == 6
    text = out.getvalue()
    assert text.count("Bad.begin") == 1 and text.count("Bad.end") == 1
    assert good.stats.steps == 3  # the healthy hook kept running


def test_stats_line_reports_rank_step_time_and_throughput():
    from sched_pass_b200.engine.engine import StepStats
    eng = FakeEngine([100, 200], R=64)
    plug = SchedPlugin(SchedPluginConfig(), stream=io.StringIO())
    eng.stats = [StepStats(6, 0, 4.0, True), StepStats(6, 0, 4.0, True)]
    line = plug.stats_line(eng)
    assert line.startswith("[sched] step=0 ") and "mode=enforce" in line
    assert "rank=0 step_ms=4.000 tok_s=1500.0" in line  # 12 tokens in 8 ms of device time
    eng.stats = []
    assert "step_ms=0.000 tok_s=0.0" in plug.stats_line(eng)
