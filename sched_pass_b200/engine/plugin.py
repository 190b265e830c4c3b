"""The per-step scheduling hooks of the serving engine.

A hook object has ``on_batch_begin(engine, plan, info)`` (before the step's
kernels are launched: bind tasks, price them, install an order, arm or
disarm the work queue, set shed budgets and the timer cadence) and
``on_batch_end(engine, plan, info, ms)`` (after the step: fold a timer
probe into the controller). ``SchedPlugin`` is the default one; the engine
runs every registered hook through ``HookRunner``, which isolates failures:
an exception in a hook is logged once per site, counted, and serving goes on
with the tables it already has (the kernels treat stale or absent tables as
the stock schedule). This is the engine-side counterpart of the reference's
SGLang plugin (python/sched_sglang_plugin.py:148-342 on_batch_begin/end,
:594-607 error isolation, :610-695 register, :698-719 effective config).

Regime gates (measured in the reference and carried over):
  * one wave (tasks <= R resident workers): ordering cannot help, the order
    is retired to identity;
  * queued (tasks > R): grouped LPT in blocks of ``lpt_block`` tasks;
  * cluster-launch-control claims are armed only when the predicted tail is
    imbalanced (max / mean cost > ``clc_imbalance``) AND the cost estimator
    is uncertain (> ``clc_resid``); otherwise static + pi;
  * L2 hints ("urgent" rows) only when the batch's KV working set exceeds L2
    (``kv_bytes_per_token`` > 0 enables the estimate).

``SchedPluginConfig`` is the typed configuration: it reads the runtime
``SCHED_*`` knobs (``from_env``) and writes them back (``to_env``), so one
object is the single source of truth for a deployment.
"""
from __future__ import annotations

import os
import sys
from dataclasses import asdict, dataclass, field, fields

import numpy as np
import torch

from . import native

_L2_BYTES = 126 * 1024 * 1024


@dataclass
class SchedPluginConfig:
    enforce: bool = True            # SCHED_ENFORCE: 0 = observe only (learn costs, install nothing)
    policy: str = "lpt"             # SCHED_POLICY: lpt | srpt | edf (controller ordering)
    timer_every: int = 8            # SCHED_TIMER_EVERY: probe cadence (0 = never)
    plan_every: int = 1             # SCHED_PLAN_EVERY: re-plan cadence (probe steps always re-plan)
    clc: str = "auto"               # SCHED_CLC_ARM: off | on | auto
    clc_resid: float = 0.75         # SCHED_CLC_RESID: estimator uncertainty to arm CLC
    clc_imbalance: float = 3.0      # SCHED_CLC_IMBALANCE: max/mean predicted cost to arm CLC
    lpt_block: int = 16             # SCHED_LPT_BLOCK
    kv_bytes_per_token: int = 0     # SCHED_KV_BYTES_PER_TOKEN: enables L2 urgency hints
    shed_fraction: float = 0.0      # SCHED_SHED_FRACTION: lowest-urgency share given a tau
    shed_ratio: float = 0.5         # SCHED_SHED_RATIO: tau = ratio * context
    stats_every: int = 512          # SCHED_STATS_EVERY: stats line cadence (0 = never)
    hooks_noop: bool = False        # SCHED_HOOKS_NOOP: hooks installed but inert
    verbose: bool = False           # SCHED_DEBUG

    _ENV = {
        "enforce": "SCHED_ENFORCE", "policy": "SCHED_POLICY", "timer_every": "SCHED_TIMER_EVERY",
        "plan_every": "SCHED_PLAN_EVERY", "clc": "SCHED_CLC_ARM", "clc_resid": "SCHED_CLC_RESID",
        "clc_imbalance": "SCHED_CLC_IMBALANCE", "lpt_block": "SCHED_LPT_BLOCK",
        "kv_bytes_per_token": "SCHED_KV_BYTES_PER_TOKEN", "shed_fraction": "SCHED_SHED_FRACTION",
        "shed_ratio": "SCHED_SHED_RATIO", "stats_every": "SCHED_STATS_EVERY",
        "hooks_noop": "SCHED_HOOKS_NOOP", "verbose": "SCHED_DEBUG",
    }

    @classmethod
    def from_engine_config(cls, ecfg) -> "SchedPluginConfig":
        clc = {"clc": "on", "auto": "auto"}.get(getattr(ecfg, "acquire", "static"), "off")
        return cls(timer_every=ecfg.timer_every, plan_every=ecfg.plan_every, clc=clc,
                   clc_resid=ecfg.clc_uncertainty, lpt_block=ecfg.lpt_block,
                   shed_fraction=ecfg.shed_fraction, shed_ratio=ecfg.shed_ratio)

    def with_env(self, env=None) -> "SchedPluginConfig":
        """A copy with every knob present in ``env`` applied (typed)."""
        env = os.environ if env is None else env
        out = SchedPluginConfig(**{f.name: getattr(self, f.name) for f in fields(self)})
        for name, key in self._ENV.items():
            if key not in env:
                continue
            cur = getattr(out, name)
            raw = env[key]
            if isinstance(cur, bool):
                val = raw not in ("0", "", "false", "False")
            elif isinstance(cur, int):
                val = int(raw)
            elif isinstance(cur, float):
                val = float(raw)
            else:
                val = raw
            setattr(out, name, val)
        if out.clc not in ("off", "on", "auto"):
            raise ValueError(f"SCHED_CLC_ARM must be off|on|auto, not {out.clc!r}")
        return out

    @classmethod
    def from_env(cls, env=None) -> "SchedPluginConfig":
        return cls().with_env(env)

    def to_env(self) -> dict:
        """The wire format: ``SCHED_*`` variables reproducing this config."""
        out = {}
        for name, key in self._ENV.items():
            v = getattr(self, name)
            out[key] = ("1" if v else "0") if isinstance(v, bool) else str(v)
        return out


class HookRunner:
    """Runs hooks with failure isolation: the first exception of each site is
    printed, later ones are only counted (and printed under SCHED_DEBUG)."""

    def __init__(self, hooks=None, stream=None):
        self.hooks = list(hooks or [])
        self.errors = 0
        self._seen: set[str] = set()
        self.stream = stream or sys.stderr

    def register(self, hook) -> None:
        if hook not in self.hooks:
            self.hooks.append(hook)

    def _error(self, where: str, exc: BaseException) -> None:
        self.errors += 1
        if where not in self._seen:
            self._seen.add(where)
            print(f"[sched] {where} hook error (control plane degraded; serving continues): {exc!r}",
                  file=self.stream)
        elif os.environ.get("SCHED_DEBUG"):
            print(f"[sched] {where} hook error: {exc!r}", file=self.stream)

    def begin(self, engine, plan, info) -> None:
        for h in self.hooks:
            try:
                h.on_batch_begin(engine, plan, info)
            except Exception as e:  # noqa: BLE001 - isolation is the point
                self._error(f"{type(h).__name__}.begin", e)

    def end(self, engine, plan, info, ms: float) -> None:
        for h in self.hooks:
            try:
                h.on_batch_end(engine, plan, info, ms)
            except Exception as e:  # noqa: BLE001
                self._error(f"{type(h).__name__}.end", e)


@dataclass
class _Stats:
    steps: int = 0
    planned: int = 0
    probes: int = 0
    clc_armed: int = 0
    orders: dict = field(default_factory=lambda: {"identity": 0, "lpt": 0, "region": 0})
    last_unc: float = float("nan")
    last_tasks: int = 0
    last_splits: int = 1


class SchedPlugin:
    """Default hook: programs the decode kernel's levers every step."""

    def __init__(self, config: SchedPluginConfig, stream=None):
        self.cfg = config
        self.stats = _Stats()
        self.stream = stream or sys.stderr
        self._probe = False

    def register(self, engine) -> "SchedPlugin":
        engine.hooks.register(self)
        print("[sched] effective config: " + self.describe(engine), file=self.stream)
        return self

    def describe(self, engine=None) -> str:
        c = self.cfg
        parts = [f"mode={'enforce' if c.enforce else 'observe'}", f"policy={c.policy}",
                 f"timer=device/every-{c.timer_every}", f"plan_every={c.plan_every}",
                 f"clc_arm={c.clc}(imbalance>{c.clc_imbalance},resid>{c.clc_resid})",
                 f"lpt_block={c.lpt_block}", f"shed={c.shed_fraction}x{c.shed_ratio}",
                 f"hints={'on' if c.kv_bytes_per_token else 'off'}"]
        if engine is not None:
            parts += [f"R={engine.R}", f"max_tasks={engine.plane.N}"]
        return " ".join(parts)

    # ------------------------------------------------------------- hooks
    def on_batch_begin(self, engine, plan, info) -> None:
        c = self.cfg
        nd, n_items = info["nd"], info["n_items"]
        self._probe = False
        info["probe"] = False
        if c.hooks_noop or not engine.ecfg.levers or nd == 0:
            return
        st = self.stats
        st.steps += 1
        hkv = engine.hkv
        n_tasks = n_items * hkv
        plane = engine.plane
        st.last_tasks, st.last_splits = n_tasks, info.get("S", 1)
        probe = c.timer_every > 0 and (engine.step_no % c.timer_every) == 0
        replan = probe or (engine.step_no % max(1, c.plan_every)) == 0
        items = engine._host("items")[:n_items * 4].reshape(-1, 4)
        if replan and c.enforce:
            st.planned += 1
            cost = native.task_costs(items, n_items, hkv)
            dec = plan.decode
            unc = engine.controller.uncertainty([r.rid for r in dec], [r.total_len for r in dec])
            st.last_unc = unc
            imbalance = float(cost.max() / max(cost.mean(), 1e-9)) if cost.size else 0.0
            queued = n_tasks > engine.R
            if c.clc == "on":
                arm_clc = True
            elif c.clc == "auto":
                arm_clc = queued and unc > c.clc_resid and imbalance > c.clc_imbalance
            else:
                arm_clc = False
            if arm_clc:
                order, kind = native.region_order(cost, engine.R, c.lpt_block), "region"
            elif queued:
                order, kind = native.grouped_lpt(cost, c.lpt_block), "lpt"
            else:
                order, kind = None, "identity"  # one wave: ordering cannot help
            st.orders[kind] += 1
            st.clc_armed += int(arm_clc)
            if order is not None:
                plane.install_order(torch.from_numpy(order), n_tasks)
            else:
                plane.set_order_size(0)
                plane.reset_order()
            # the decode kernel is persistent for every acquisition mode:
            # arming only selects whether its claims run
            plane.set_num_tasks(n_tasks if engine.ecfg.acquire in ("ticket", "clc", "auto") else 0)
            self._hints(engine, plan, items, n_items)
        if c.enforce and (c.shed_fraction > 0 or any(r.tau for r in plan.decode)):
            self._shed(engine, plan, items, n_items)
        plane.set_timer_enabled(probe)
        if probe:
            plane.clear_timer()
        plane.push()
        self._probe = probe
        info["probe"] = probe  # per step: the engine may begin step k + 1 before it ends step k

    def on_batch_end(self, engine, plan, info, ms: float) -> None:
        c = self.cfg
        if info.get("probe", self._probe) and info["nd"] > 0:
            self._fold_probe(engine, plan, info)
            self.stats.probes += 1
        self._probe = False
        if c.stats_every > 0 and self.stats.steps and engine.step_no % c.stats_every == 0:
            print(self.stats_line(engine), file=self.stream)

    # ------------------------------------------------------------- pieces
    def _shed(self, engine, plan, items, n_items) -> None:
        """tau rows: a request's own budget (``Request.tau``) when it has one,
        else ``shed_ratio`` x context for the lowest-urgency ``shed_fraction``.
        The budget is written back to the request so the tiered KV store
        knows which pages the kernel will not read."""
        c = self.cfg
        dec = plan.decode
        k = int(len(dec) * c.shed_fraction)
        low = set(sorted((i for i in range(len(dec)) if not dec[i].tau), key=lambda i: dec[i].urgency)[:k])
        for i in low:
            dec[i].tau = max(1, int(c.shed_ratio * dec[i].total_len))
        if not any(r.tau for r in dec):
            return
        hkv = engine.hkv
        tau = np.zeros(n_items * hkv, dtype=np.int64)
        for it in range(n_items):
            r = dec[int(items[it, 0])]
            if r.tau:
                tau[it * hkv:(it + 1) * hkv] = min(int(r.tau), r.total_len)
        engine.plane.set_rows(tau=np.minimum(tau, 0xFFFF), n=n_items * hkv)

    def _hints(self, engine, plan, items, n_items) -> None:
        """Urgency rows (q) only pay when the batch's KV does not fit in L2."""
        c = self.cfg
        if not c.kv_bytes_per_token:
            return
        dec = plan.decode
        footprint = sum(r.total_len for r in dec) * c.kv_bytes_per_token
        if footprint <= _L2_BYTES:
            return
        hkv = engine.hkv
        q = np.zeros(n_items * hkv, dtype=np.float32)
        for it in range(n_items):
            q[it * hkv:(it + 1) * hkv] = dec[int(items[it, 0])].urgency
        engine.plane.set_rows(q=q, n=n_items * hkv)

    def _fold_probe(self, engine, plan, info) -> None:
        """Per-request cycles of a probe step into the controller. The
        engine snapshots the timer rows right after the step's forward
        (``info["timer"]``, host memory) and keeps the step's work items and
        KV lengths in ``info``, because the next step may already be
        planned (and the timer cleared) when this runs."""
        hkv = engine.hkv
        n_items = info["n_items"]
        timer = info.get("timer")
        if timer is None:
            timer = engine.plane.timer_t[: n_items * hkv].cpu()
        cyc = timer[: n_items * hkv].view(n_items, hkv).sum(1).numpy()
        items = info.get("items")
        if items is None:
            items = engine._host("items")[: n_items * 4].reshape(-1, 4)
        per_req = np.zeros(info["nd"], dtype=np.float64)
        np.add.at(per_req, items[:n_items, 0], cyc)
        dec = plan.decode
        lens = info.get("kv_lens")
        engine.controller.observe([r.rid for r in dec], lens if lens is not None else [r.total_len for r in dec],
                                  per_req[: len(dec)].tolist())

    def stats_line(self, engine) -> str:
        """The periodic stats line: the reference's fields, then this rank,
        the device time of its last step and its decode tokens per second of
        device time over the last 64 steps (under TP every rank prints its
        own line; the box's throughput is any rank's, since all decode the
        same tokens)."""
        s = self.stats
        recent = list(getattr(engine, "stats", None) or [])[-64:]
        dev_ms = sum(st.device_ms for st in recent)
        tok_s = sum(st.n_decode for st in recent) / (dev_ms / 1e3) if dev_ms > 0 else 0.0
        tp = getattr(engine, "tp", None)
        rank = tp.rank if tp is not None else 0
        return (f"[sched] step={engine.step_no} tasks={s.last_tasks} split={s.last_splits} R={engine.R} "
                f"planned={s.planned} probes={s.probes} unc={s.last_unc:.3f} clc_armed={s.clc_armed} "
                f"orders={s.orders} errors={engine.hooks.errors} "
                f"mode={'enforce' if self.cfg.enforce else 'observe'} "
                f"rank={rank} step_ms={recent[-1].device_ms if recent else 0.0:.3f} tok_s={tok_s:.1f}")

    def as_dict(self) -> dict:
        return asdict(self.cfg)
