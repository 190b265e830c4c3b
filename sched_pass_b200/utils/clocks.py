"""GPU clock / throttle sampling during a timed region (nvidia-smi, read-only)."""
from __future__ import annotations

import os
import shutil
import statistics
import subprocess
import tempfile

QUERY = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
REASONS = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")


class ClockSampler:
    """Starts ``nvidia-smi -lms`` in the background; ``stop()`` returns a
    summary {sm_mhz (median under load), sm_max_mhz, reasons[], samples}.
    The default period of 20 ms gives a window of a tenth of a second a few
    samples."""

    def __init__(self, gpu_index: int | None = None, period_ms: int = 20, log_path: str | None = None):
        self.gpu = gpu_index
        self.period = period_ms
        self.proc = None
        self.path = log_path or tempfile.mktemp(prefix="clocks_", suffix=".csv")

    def start(self) -> "ClockSampler":
        exe = shutil.which("nvidia-smi")
        if exe is None:
            return self
        cmd = [exe, f"--query-gpu={QUERY}", "--format=csv,noheader,nounits", f"-lms={self.period}"]
        if self.gpu is not None:
            cmd.insert(1, f"-i={self.gpu}")
        self._f = open(self.path, "w")
        self.proc = subprocess.Popen(cmd, stdout=self._f, stderr=subprocess.DEVNULL)
        return self

    def stop(self, window: tuple[float, float] | None = None) -> dict:
        """Stop sampling and summarise. ``window`` = (t0, t1) in
        ``time.time()`` seconds keeps the samples taken inside it (plus the
        nearest one on each side, so a window shorter than the period still
        has its neighbours)."""
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"], "samples": 0}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self._f.close()
        rows = []
        with open(self.path) as f:
            for line in f:
                row = parse_line(line)
                if row is not None:
                    rows.append(row)
        return summarize(rows, window)


def parse_line(line: str):
    """(unix time or None, sm MHz, max sm MHz, {reason: active}) of one CSV
    line of ``QUERY``, or None if it does not parse."""
    import datetime
    parts = [p.strip() for p in line.split(",")]
    if len(parts) < 10:
        return None
    try:
        sm, smax = float(parts[2]), float(parts[3])
    except ValueError:
        return None
    try:
        ts = datetime.datetime.strptime(parts[0], "%Y/%m/%d %H:%M:%S.%f").timestamp()
    except ValueError:
        ts = None
    active = {name: val.lower() == "active" for name, val in zip(REASONS, parts[6:10])}
    return ts, sm, smax, active


def summarize(rows: list, window: tuple[float, float] | None = None) -> dict:
    if window is not None and rows and all(r[0] is not None for r in rows):
        t0, t1 = window
        inside = [i for i, r in enumerate(rows) if t0 <= r[0] <= t1]
        before = [i for i, r in enumerate(rows) if r[0] < t0]
        after = [i for i, r in enumerate(rows) if r[0] > t1]
        keep = sorted(set(inside + before[-1:] + after[:1]))
        rows = [rows[i] for i in keep]
    if not rows:
        return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
    sm = [r[1] for r in rows]
    reasons = sorted({name for r in rows for name, on in r[3].items() if on})
    loaded = [x for x in sm if x > 0.5 * max(sm)] or sm
    return {"sm_mhz": statistics.median(loaded), "sm_max_mhz": max(r[2] for r in rows), "reasons": reasons,
            "samples": len(rows)}
