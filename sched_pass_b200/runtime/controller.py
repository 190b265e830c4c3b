"""Closed-loop scheduling controller: estimate task costs, order the batch,
damp order changes.

Public surface and semantics of the reference controller (jc-su/sched-pass
python/sched_controller.py:58-177): ``observe``, ``observe_step``,
``predict_one``, ``gamma``, ``uncertainty``, ``order``, ``step``, plus
``forget`` for finished requests. The implementation is array-based: a
step's batch is folded in and ordered with numpy operations, not per-request
Python loops.

Estimation. Each kernel family (``"decode"`` by default; a caller may keep
``"prefill"`` or any other family apart) has a ``CostModel``: the normal
equations of a least-squares line ``cycles = slope * kv_len + intercept``
kept as a 2 x 2 Gram matrix and a moment vector, updated with a whole batch
at once (``decay`` < 1 forgets old batches geometrically; 1 keeps plain least
squares). What the line misses for one request is an exponentially weighted
residual held in a slot table (request id -> row of a numpy array, rows
reused after ``forget``). ``gamma`` is an exponentially weighted ratio of
measured to predicted step time, for a pricing layer; the serving loop does
not consume it.

Ordering. LPT (longest first: makespan), SRPT (shortest first: mean
latency) or EDF (least slack first: deadlines), as a stable argsort of the
predictions, so ties keep batch order.

Damping. A new order is published only if it lowers the predicted total
completion time (sum over tasks of the time at which each finishes when
served in that order) by more than ``deadband`` of the new total; otherwise
the previous order of a same-sized batch stays, so noise does not churn the
published order.
"""
from __future__ import annotations

import numpy as np


class CostModel:
    """Least-squares line y = slope * x + intercept over batches of (x, y),
    through its normal equations: ``gram`` = sum of [x, 1]^T [x, 1] and
    ``moment`` = sum of y [x, 1]. Fewer than two distinct x: the line through
    the origin and the mean point (slope 1 with no data)."""

    def __init__(self, decay: float = 1.0):
        self.decay = float(decay)
        self.gram = np.zeros((2, 2))
        self.moment = np.zeros(2)

    @property
    def count(self) -> float:
        return float(self.gram[1, 1])

    def add(self, x, y) -> None:
        x = np.asarray(x, dtype=np.float64).ravel()
        y = np.asarray(y, dtype=np.float64).ravel()
        if x.size == 0:
            return
        if self.decay != 1.0:
            self.gram *= self.decay
            self.moment *= self.decay
        self.gram += np.array([[x @ x, x.sum()], [x.sum(), float(x.size)]])
        self.moment += np.array([x @ y, y.sum()])

    def coeffs(self) -> tuple[float, float]:
        (sxx, sx), (_, n) = self.gram
        sxy, sy = self.moment
        det = sxx * n - sx * sx
        # a line needs two distinct x: the determinant is n^2 var(x), compare it
        # with the scale of the data so rounding noise is not mistaken for spread
        if n >= 2 and det > 1e-12 * max(sxx * n, 1e-300):
            slope, intercept = np.linalg.solve(self.gram, self.moment)
            return float(slope), float(intercept)
        return (float(sy / sx) if sx > 0 else 1.0), 0.0

    def predict(self, x) -> np.ndarray:
        a, b = self.coeffs()
        return np.maximum(a * np.asarray(x, dtype=np.float64) + b, 0.0)


class ResidualTable:
    """Per-request residuals in a growable array, addressed through a map from
    request id to row; rows of forgotten requests are reused."""

    def __init__(self, capacity: int = 256):
        self.value = np.zeros(capacity)
        self.row: dict = {}
        self._free: list = []

    def __contains__(self, rid) -> bool:
        return rid in self.row

    def rows(self, rids, create: bool) -> np.ndarray:
        """Rows of ``rids`` (-1 for unknown ids unless ``create``)."""
        out = np.empty(len(rids), dtype=np.int64)
        for i, rid in enumerate(rids):
            r = self.row.get(rid)
            if r is None and create:
                if self._free:
                    r = self._free.pop()
                else:
                    r = len(self.row)
                    if r >= self.value.size:
                        self.value = np.concatenate([self.value, np.zeros(self.value.size)])
                self.value[r] = 0.0
                self.row[rid] = r
            out[i] = -1 if r is None else r
        return out

    def get(self, rid, default: float = 0.0) -> float:
        r = self.row.get(rid)
        return default if r is None else float(self.value[r])

    def drop(self, rids) -> None:
        for rid in rids:
            r = self.row.pop(rid, None)
            if r is not None:
                self._free.append(r)


class SchedControlPlane:
    """Estimator + policy for a batch of (request id, KV length) tasks."""

    def __init__(self, policy: str = "lpt", ewma: float = 0.25, deadband: float = 0.02, decay: float = 1.0):
        if policy not in ("lpt", "srpt", "edf"):
            raise ValueError(f"unknown policy {policy!r}")
        self.policy = policy
        self.ewma = float(ewma)        # smoothing of residuals and gamma
        self.deadband = float(deadband)  # relative gain needed to publish a new order
        self.decay = float(decay)      # forgetting factor of the cost lines (1: plain least squares)
        self.models: dict[str, CostModel] = {}
        self.residuals: dict[str, ResidualTable] = {}
        self._gamma = 1.0
        self._published: np.ndarray | None = None

    # ---- estimation ------------------------------------------------------
    def model(self, family: str = "decode") -> CostModel:
        m = self.models.get(family)
        if m is None:
            m = self.models[family] = CostModel(self.decay)
            self.residuals[family] = ResidualTable()
        return m

    def coeffs(self, family: str = "decode") -> tuple[float, float]:
        """(slope, intercept) of a family's cost line."""
        return self.model(family).coeffs()

    def observe(self, rids, kv_lens, cycles, family: str = "decode") -> None:
        """Fold one step's measured per-task cycles (0 = not measured) into
        the family's line, then move each measured request's residual towards
        what the updated line misses for it."""
        cyc = np.asarray(cycles, dtype=np.float64).ravel()
        keep = np.flatnonzero(cyc > 0)
        if keep.size == 0:
            return
        x = np.asarray(kv_lens, dtype=np.float64).ravel()[keep]
        y = cyc[keep]
        m = self.model(family)
        m.add(x, y)
        table = self.residuals[family]
        rows = table.rows([rids[i] for i in keep], create=True)
        table.value[rows] += self.ewma * ((y - m.predict(x)) - table.value[rows])

    def observe_step(self, predicted_makespan: float, measured_makespan: float) -> None:
        """Congestion index: gamma > 1 when steps run slower than the model
        predicts (co-runners taking bandwidth). Exposed for a pricing layer
        that sets lambda; the serving loop does not consume it."""
        if predicted_makespan > 0 and measured_makespan > 0:
            self._gamma += self.ewma * (measured_makespan / predicted_makespan - self._gamma)

    def predict(self, rids, kv_lens, family: str = "decode") -> np.ndarray:
        """Predicted cycles of a batch, residuals included (never negative)."""
        a, b = self.model(family).coeffs()
        base = a * np.asarray(kv_lens, dtype=np.float64) + b
        if rids is not None:
            table = self.residuals[family]
            rows = table.rows(list(rids), create=False)
            base = base + np.where(rows >= 0, table.value[np.maximum(rows, 0)], 0.0)
        return np.maximum(base, 0.0)

    def predict_one(self, kv_len: float, rid=None, family: str = "decode") -> float:
        t = self.model(family).predict([kv_len])[0]
        if rid is not None:
            t = max(t + self.residuals[family].get(rid), 0.0)
        return float(t)

    def forget(self, rids, family: str | None = None) -> None:
        """Drop the residual state of finished requests (every family by default)."""
        for f, table in self.residuals.items():
            if family is None or f == family:
                table.drop(rids)

    @property
    def gamma(self) -> float:
        return self._gamma

    def uncertainty(self, rids, kv_lens, family: str = "decode") -> float:
        """Mean |residual| over mean prediction for a batch, where a request
        never observed counts its whole prediction as doubt. High values are
        the signal that arms late-binding acquisition (which needs no
        prediction to balance the batch)."""
        if len(rids) == 0:
            return 1.0
        pred = self.model(family).predict(kv_lens)
        mean_pred = float(pred.mean())
        if mean_pred <= 0:
            return 1.0
        table = self.residuals[family]
        rows = table.rows(list(rids), create=False)
        doubt = np.where(rows >= 0, np.abs(table.value[np.maximum(rows, 0)]), pred)
        return float(doubt.mean()) / mean_pred

    # ---- ordering ----------------------------------------------------------
    @staticmethod
    def completion_total(t_hat: np.ndarray, order: np.ndarray) -> float:
        """Total completion time of serving ``order`` one task after another:
        the k-th task served is waited for by the n - k tasks from it on."""
        n = order.size
        return float(np.arange(n, 0, -1, dtype=np.float64) @ t_hat[order]) if n else 0.0

    def order(self, rids, kv_lens, deadlines=None, elapsed=None, family: str = "decode") -> list:
        """Batch indices in serving order under the policy, damped by the
        dead-band against the previously published order."""
        t_hat = self.predict(rids, kv_lens, family)
        n = t_hat.size
        if self.policy == "lpt":
            new = np.argsort(-t_hat, kind="stable")
        elif self.policy == "srpt":
            new = np.argsort(t_hat, kind="stable")
        else:
            if deadlines is None:
                raise ValueError("the edf policy needs deadlines")
            slack = np.asarray(deadlines, dtype=np.float64) - t_hat
            if elapsed is not None:
                slack = slack - np.asarray(elapsed, dtype=np.float64)
            new = np.argsort(slack, kind="stable")
        prev = self._published
        if prev is not None and prev.size == n:
            cand = self.completion_total(t_hat, new)
            if self.completion_total(t_hat, prev) - cand < self.deadband * max(cand, 1e-9):
                return prev.tolist()
        self._published = new
        return new.tolist()

    # ---- one serving step ------------------------------------------------
    def step(self, plane, rids, kv_lens, cycles=None, deadlines=None, elapsed=None) -> list:
        """Fold the step's measurements, order the batch and program the
        plane (order, task count, publication). Returns the order."""
        if cycles is not None:
            self.observe(rids, kv_lens, cycles)
        order = self.order(rids, kv_lens, deadlines, elapsed)
        plane.set_order(order)
        plane.set_num_tasks(len(order))
        plane.push()
        return order
