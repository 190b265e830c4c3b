"""GPU clock / throttle sampling during a timed region (nvidia-smi, read-only)."""
from __future__ import annotations

import os
import shutil
import statistics
import subprocess
import tempfile

QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
REASONS = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")


class ClockSampler:
    """Starts ``nvidia-smi -lms`` in the background; ``stop()`` returns a
    summary {sm_mhz (median under load), sm_max_mhz, reasons[], samples}."""

    def __init__(self, gpu_index: int | None = None, period_ms: int = 200, log_path: str | None = None):
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

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"], "samples": 0}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self._f.close()
        sm, smax, reasons = [], [], set()
        with open(self.path) as f:
            for line in f:
                parts = [p.strip() for p in line.split(",")]
                if len(parts) < 9:
                    continue
                try:
                    sm.append(float(parts[1]))
                    smax.append(float(parts[2]))
                except ValueError:
                    continue
                for name, val in zip(REASONS, parts[5:9]):
                    if val.lower() == "active":
                        reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        loaded = [s for s in sm if s > 0.5 * max(sm)] or sm
        return {"sm_mhz": statistics.median(loaded), "sm_max_mhz": max(smax), "reasons": sorted(reasons),
                "samples": len(sm)}
