"""Summarise an Nsight Compute capture into the markdown rows kept under
``profiles/``: one row per captured launch with its duration, DRAM traffic
and throughput, tensor-pipe activity, occupancy, registers and the three
largest warp-stall reasons, plus the achieved bandwidth as a fraction of the
measured HBM copy rate (``MEASURED_PEAKS.json``).

Input is the raw-page CSV (``ncu -i rep.ncu-rep --page raw --csv``: a header
row of metric names, a row of units, then one row per launch), given as a
file, on stdin, or produced here from a ``.ncu-rep`` path. Only counters are
read (no source or SASS page).

    ncu -i prof.ncu-rep --page raw --csv > prof.csv
    python -m sched_pass_b200.benchmarks.ncu_summary prof.csv [--bytes N] [--flops F]

``--bytes`` / ``--flops``: the algorithmic bytes / FLOPs of one launch, to
report achieved = algorithmic / duration beside the counter-derived traffic.
"""
from __future__ import annotations

import argparse
import csv
import io
import subprocess
import sys

from .common import measured_peaks

METRICS = {
    "time": "gpu__time_duration.sum",
    "dram_read": "dram__bytes_read.sum",
    "dram_write": "dram__bytes_write.sum",
    "dram_pct": "gpu__dram_throughput.avg.pct_of_peak_sustained_elapsed",
    "tensor_pct": "sm__pipe_tensor_cycles_active.avg.pct_of_peak_sustained_active",
    "warps_pct": "sm__warps_active.avg.pct_of_peak_sustained_active",
    "regs": "launch__registers_per_thread",
    "grid": "launch__grid_size",
    "block": "launch__block_size",
}
STALL_PREFIX = "smsp__average_warps_issue_stalled_"
TIME_SCALE = {"nsecond": 1e-9, "usecond": 1e-6, "msecond": 1e-3, "second": 1.0, "ns": 1e-9, "us": 1e-6}
BYTE_SCALE = {"byte": 1.0, "Kbyte": 1e3, "Mbyte": 1e6, "Gbyte": 1e9, "KB": 1e3, "MB": 1e6, "GB": 1e9}


def number(text: str):
    t = (text or "").strip().replace(",", "")
    if not t or t in ("n/a", "N/A"):
        return None
    try:
        return float(t)
    except ValueError:
        return None


def parse(text: str) -> list[dict]:
    """Rows of the raw CSV as {metric: (value, unit)} plus the kernel name."""
    rows = list(csv.reader(io.StringIO(text)))
    rows = [r for r in rows if r and not r[0].startswith("==")]  # ncu banner lines
    if len(rows) < 2:
        return []
    head, units = rows[0], rows[1]
    out = []
    for r in rows[2:]:
        rec = {"kernel": r[head.index("Kernel Name")] if "Kernel Name" in head else "?"}
        for i, name in enumerate(head):
            if i < len(r):
                rec[name] = (r[i], units[i] if i < len(units) else "")
        out.append(rec)
    return out


def value(rec: dict, name: str, scale: dict | None = None):
    if name not in rec:
        return None
    v = number(rec[name][0])
    if v is None or scale is None:
        return v
    return v * scale.get(rec[name][1].strip(), 1.0)


def summarize(rec: dict, peaks: dict, alg_bytes: float | None = None, alg_flops: float | None = None) -> dict:
    t = value(rec, METRICS["time"], TIME_SCALE)
    rd = value(rec, METRICS["dram_read"], BYTE_SCALE) or 0.0
    wr = value(rec, METRICS["dram_write"], BYTE_SCALE) or 0.0
    stalls = sorted(((number(v[0]) or 0.0, k[len(STALL_PREFIX):].split(".")[0].replace("_per_issue_active", ""))
                     for k, v in rec.items() if k.startswith(STALL_PREFIX) and k.endswith(".ratio")),
                    reverse=True)[:3]
    s = {"kernel": rec["kernel"], "us": None if t is None else t * 1e6,
         "dram_MB": (rd + wr) / 1e6, "dram_pct": value(rec, METRICS["dram_pct"]),
         "tensor_pct": value(rec, METRICS["tensor_pct"]), "warps_pct": value(rec, METRICS["warps_pct"]),
         "regs": value(rec, METRICS["regs"]), "stalls": [n for v, n in stalls if v > 0]}
    if t:
        s["dram_GBps"] = (rd + wr) / t / 1e9
        s["frac_hbm_of_measured"] = s["dram_GBps"] / peaks["hbm_gbs"]
        if alg_bytes:
            s["alg_GBps"] = alg_bytes / t / 1e9
        if alg_flops:
            s["alg_TFLOPs"] = alg_flops / t / 1e12
            s["frac_bf16_of_measured"] = s["alg_TFLOPs"] / peaks["bf16_tflops"]
    return s


def markdown(summaries: list[dict]) -> str:
    cols = [("kernel", "kernel"), ("us", "us"), ("dram_MB", "DRAM MB"), ("dram_GBps", "DRAM GB/s"),
            ("frac_hbm_of_measured", "of measured HBM"), ("dram_pct", "dram %"), ("tensor_pct", "tensor %"),
            ("warps_pct", "warps active %"), ("regs", "regs"), ("alg_TFLOPs", "alg TFLOP/s"),
            ("stalls", "top stalls")]
    cols = [c for c in cols if any(s.get(c[0]) not in (None, []) for s in summaries)]

    def fmt(v):
        if isinstance(v, float):
            return f"{v:.3g}" if abs(v) < 1000 else f"{v:.0f}"
        if isinstance(v, list):
            return ", ".join(v)
        return "" if v is None else str(v)

    lines = ["| " + " | ".join(h for _, h in cols) + " |", "|" + "---|" * len(cols)]
    for s in summaries:
        lines.append("| " + " | ".join(fmt(s.get(k)) for k, _ in cols) + " |")
    return "\n".join(lines)


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("src", nargs="?", default="-", help="raw CSV, .ncu-rep, or - for stdin")
    ap.add_argument("--bytes", type=float, default=None, help="algorithmic bytes of one launch")
    ap.add_argument("--flops", type=float, default=None, help="algorithmic FLOPs of one launch")
    a = ap.parse_args(argv)
    if a.src == "-":
        text = sys.stdin.read()
    elif a.src.endswith(".ncu-rep"):
        text = subprocess.run(["ncu", "-i", a.src, "--page", "raw", "--csv"], capture_output=True, text=True,
                              check=True).stdout
    else:
        with open(a.src) as f:
            text = f.read()
    peaks = measured_peaks()
    sums = [summarize(r, peaks, a.bytes, a.flops) for r in parse(text)]
    print(markdown(sums))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
