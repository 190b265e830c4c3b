"""Closed-loop scheduling controller: estimate, order, damp.

Same public surface as the reference controller (python/sched_controller.py
:58-177 of jc-su/sched-pass): ``observe``, ``observe_step``, ``predict_one``,
``gamma``, ``uncertainty``, ``order``, ``step``.

1. Estimation -- per kernel family an online least-squares line
   ``t = alpha * kv_len + beta`` over measured per-task cycles (the woven
   timer), a per-request exponentially weighted residual for what the line
   misses, and a congestion index gamma (measured / predicted step time).
2. Ordering -- LPT (makespan), SRPT (mean latency) or EDF (deadlines) by
   sorting the predictions.
3. Damping -- a new order replaces the published one only when it improves
   the order-dependent quality score (total completion time) by more than a
   dead-band, so small fluctuations do not churn the order.

Pure Python; drives anything with ``set_order``/``set_num_tasks``/``push``.
"""
from __future__ import annotations

from dataclasses import dataclass, field


@dataclass
class LineFit:
    """Running sums for an ordinary least-squares line y = a x + b."""

    n: int = 0
    sx: float = 0.0
    sy: float = 0.0
    sxx: float = 0.0
    sxy: float = 0.0

    def add(self, x: float, y: float) -> None:
        self.n += 1
        self.sx += x
        self.sy += y
        self.sxx += x * x
        self.sxy += x * y

    def coeffs(self) -> tuple[float, float]:
        """(slope, intercept). With fewer than two distinct x the line is
        taken through the origin (proportional cost), or slope 1 if empty."""
        det = self.n * self.sxx - self.sx * self.sx
        if self.n >= 2 and det > 0:
            a = (self.n * self.sxy - self.sx * self.sy) / det
            return a, (self.sy - a * self.sx) / self.n
        return ((self.sy / self.sx) if self.sx > 0 else 1.0), 0.0


@dataclass
class SchedControlPlane:
    policy: str = "lpt"       # lpt | srpt | edf
    ewma: float = 0.25        # smoothing of residuals and gamma
    deadband: float = 0.02    # minimum relative gain to publish a new order
    _fit: LineFit = field(default_factory=LineFit)
    _resid: dict = field(default_factory=dict)
    _gamma: float = 1.0
    _last_order: list = field(default_factory=list)

    # ---- estimation ------------------------------------------------------
    def observe(self, rids, kv_lens, cycles) -> None:
        """Fold one step's measured cycles (0 = not measured) into the model."""
        for rid, ln, cy in zip(rids, kv_lens, cycles):
            cy = float(cy)
            if cy <= 0.0:
                continue
            self._fit.add(float(ln), cy)
            err = cy - self.predict_one(ln)
            prev = self._resid.get(rid, 0.0)
            self._resid[rid] = prev + self.ewma * (err - prev)

    def observe_step(self, predicted_makespan: float, measured_makespan: float) -> None:
        """Congestion index: gamma > 1 when the step ran slower than the
        model predicts (co-runners taking bandwidth). Exposed for a pricing
        layer that sets lambda; the serving loop does not consume it."""
        if predicted_makespan > 0 and measured_makespan > 0:
            ratio = measured_makespan / predicted_makespan
            self._gamma += self.ewma * (ratio - self._gamma)

    def predict_one(self, kv_len: float, rid=None) -> float:
        a, b = self._fit.coeffs()
        t = a * float(kv_len) + b
        if rid is not None:
            t += self._resid.get(rid, 0.0)
        return t if t > 0.0 else 0.0

    def forget(self, rids) -> None:
        """Drop the residual state of finished requests."""
        for r in rids:
            self._resid.pop(r, None)

    @property
    def gamma(self) -> float:
        return self._gamma

    def uncertainty(self, rids, kv_lens) -> float:
        """Mean |residual| over mean prediction for a batch. Requests never
        observed count a full prediction of doubt. This is the signal that
        arms late-binding acquisition (which does not need predictions)."""
        if not rids:
            return 1.0
        preds = [self.predict_one(ln) for ln in kv_lens]
        doubt = [abs(self._resid[r]) if r in self._resid else p for r, p in zip(rids, preds)]
        mp = sum(preds) / len(preds)
        return (sum(doubt) / len(doubt)) / mp if mp > 0 else 1.0

    # ---- ordering ----------------------------------------------------------
    def order(self, rids, kv_lens, deadlines=None, elapsed=None) -> list:
        t_hat = [self.predict_one(ln, rid) for rid, ln in zip(rids, kv_lens)]
        n = len(t_hat)
        if self.policy == "lpt":
            new = sorted(range(n), key=lambda i: -t_hat[i])
        elif self.policy == "srpt":
            new = sorted(range(n), key=lambda i: t_hat[i])
        elif self.policy == "edf":
            if deadlines is None:
                raise ValueError("edf needs deadlines")
            el = elapsed if elapsed is not None else [0.0] * n
            new = sorted(range(n), key=lambda i: deadlines[i] - el[i] - t_hat[i])
        else:
            raise ValueError(f"unknown policy {self.policy!r}")
        if len(self._last_order) == n:
            keep = self._span(t_hat, self._last_order)
            cand = self._span(t_hat, new)
            if keep - cand < self.deadband * max(cand, 1e-9):
                return self._last_order
        self._last_order = new
        return new

    @staticmethod
    def _span(t_hat, order) -> float:
        """Total completion time of serving ``order`` one task at a time: the
        sum of prefix sums. Unlike the makespan it depends on the order, so
        the dead-band reacts to real ranking changes."""
        total = acc = 0.0
        for i in order:
            acc += t_hat[i]
            total += acc
        return total

    # ---- one serving step ------------------------------------------------------
    def step(self, plane, rids, kv_lens, cycles=None, deadlines=None, elapsed=None) -> list:
        if cycles is not None:
            self.observe(rids, kv_lens, cycles)
        order = self.order(rids, kv_lens, deadlines, elapsed)
        plane.set_order(order)
        plane.set_num_tasks(len(order))
        plane.push()
        return order
