"""tcgen05 GEMM vs the HBM / tensor roofline on Llama-3-8B projection shapes.

For each (T tokens, N, K): our kernel's median time, the weight-streaming
bandwidth it achieves (bytes of W + X + Y over time), its TFLOP/s, and the
same shape through torch.matmul (cuBLAS) for reference. L2 is flushed
between iterations. Prints one JSON object per shape.
"""
from __future__ import annotations

import argparse
import json

import torch

from .. import ops
from .common import L2Flusher, measured_peaks, time_fn

SHAPES = {"qkv": (6144, 4096), "o": (4096, 4096), "gate_up": (28672, 4096), "down": (4096, 14336),
          "lm_head": (128256, 4096)}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--tokens", default="1,16,64,128,256,2048")
    ap.add_argument("--shapes", default=",".join(SHAPES))
    ap.add_argument("--iters", type=int, default=20)
    args = ap.parse_args()
    peaks = measured_peaks()
    flush = L2Flusher("cuda")
    for name in args.shapes.split(","):
        N, K = SHAPES[name]
        w = (torch.randn(N, K, device="cuda") / 64).to(torch.bfloat16)
        for T in (int(t) for t in args.tokens.split(",")):
            x = torch.randn(T, K, device="cuda").to(torch.bfloat16)
            y = torch.empty(T, N // 2 if name == "gate_up" else N, dtype=torch.bfloat16, device="cuda")
            swiglu = name == "gate_up"
            ms = time_fn(lambda: ops.linear(x, w, y, swiglu=swiglu), args.iters, flush=flush)
            ms_cublas = time_fn(lambda: torch.matmul(x, w.t()), args.iters, flush=flush)
            byts = 2 * (N * K + T * K + T * y.shape[1])
            flops = 2 * T * N * K
            rec = {"shape": name, "T": T, "N": N, "K": K, "us": round(ms * 1e3, 2),
                   "GBps": round(byts / ms / 1e6, 1), "TFLOPs": round(flops / ms / 1e9, 1),
                   "frac_hbm_of_measured": round(byts / ms / 1e6 / peaks["hbm_gbs"], 3),
                   "frac_bf16_of_measured": round(flops / ms / 1e9 / peaks["bf16_tflops"], 3),
                   "cublas_us": round(ms_cublas * 1e3, 2),
                   "speedup_vs_cublas": round(ms_cublas / ms, 3)}
            print(json.dumps(rec), flush=True)
    ops.check_status()


if __name__ == "__main__":
    main()
