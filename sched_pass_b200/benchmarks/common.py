"""Device timing helpers shared by the microbenchmarks."""
from __future__ import annotations

import json
import os

import torch

L2_FLUSH_BYTES = 256 << 20  # > 126 MB L2


class L2Flusher:
    def __init__(self, device):
        self.buf = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.int32, device=device)

    def __call__(self):
        self.buf.fill_(1)


def time_fn(fn, iters: int = 20, warmup: int = 5, flush: L2Flusher | None = None) -> float:
    """Median device time (ms) of fn over ``iters`` launches, CUDA events on
    the current stream, optional L2 flush between iterations."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    times = []
    for _ in range(iters):
        if flush is not None:
            flush()
        s = torch.cuda.Event(enable_timing=True)
        e = torch.cuda.Event(enable_timing=True)
        s.record()
        fn()
        e.record()
        e.synchronize()
        times.append(s.elapsed_time(e))
    times.sort()
    return times[len(times) // 2]


def measured_peaks() -> dict:
    path = os.path.join(os.path.dirname(__file__), "..", "..", "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return json.load(f)
    except OSError:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "fallback": True}
