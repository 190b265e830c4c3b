"""One gloo rank of the fused all-reduce protocol emulation
(sched_pass_b200/parallel/protocol.py). Scenario from argv[1]; prints one
``PROTOJSON {...}`` line."""
import faulthandler
import datetime
import json
import os
import sys

import numpy as np
import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))))
from sched_pass_b200.parallel import protocol as P  # noqa: E402


def inputs(rank, call, T, K, N):
    g = torch.Generator().manual_seed(1000 * call + rank)
    x = torch.randn(T, K, generator=g).to(torch.bfloat16)
    w = (torch.randn(N, K, generator=g) / K ** 0.5).to(torch.bfloat16)
    return x, w


def expected(world, call, T, K, N):
    parts = np.stack([P.to_bf16_bits(a.float() @ b.float().t()) for a, b in
                      (inputs(r, call, T, K, N) for r in range(world))])
    fp32 = sum(a.float() @ b.float().t() for a, b in (inputs(r, call, T, K, N) for r in range(world)))
    return parts, fp32


faulthandler.enable()  # a native crash prints the Python stack of every thread


def run_lines(scen, fab, rank, world, out):
    """Scenarios of the decode-size line exchange. One emulator (one epoch
    state) per process, as the kernel keeps one per rank."""
    import time
    lar = P.EmulatedLineAllReduce(fab, budget_s=1.5 if scen != "ll_drop" else 0.5)
    bad, statuses, call = [], [], 0

    def check(T, K, N, **kw):
        nonlocal call
        x, w = inputs(rank, call, T, K, N)
        y, st = lar(x, w, seed=rank * 7919 + call, **kw)
        parts, fp32 = expected(world, call, T, K, N)
        yb = y.view(torch.int16).numpy().view(np.uint16)
        if not np.array_equal(yb, P.reduce_rank_order(parts)):
            bad.append([call, T, N, lar.multicast, "bits"])
        err = (y.float() - fp32).abs().max().item() / max(1e-6, fp32.abs().max().item())
        if err > 2e-2:
            bad.append([call, T, N, f"err {err:.3g}"])
        statuses.append(st)
        call += 1

    shapes = [(1, 64, 128), (5, 64, 256), (16, 128, 128), (33, 64, 256), (48, 32, 256), (2, 64, 64)]
    if scen == "ll_exact":
        for mc in (False, True):
            lar.multicast = mc
            for T, K, N in shapes:
                check(T, K, N)
    elif scen == "ll_torn":
        for mc in (False, True):
            lar.multicast = mc
            for T, K, N in shapes:
                check(T, K, N, torn=True)
    elif scen == "ll_skew":
        for mc in (False, True):
            lar.multicast = mc
            for i in range(3):
                check(40, 64, 256, stall_s=0.3 if rank == world - 1 else 0.0)
    elif scen == "ll_drop":
        x, w = inputs(rank, 0, 40, 64, 128)
        t0 = time.monotonic()
        _, st = lar(x, w, drop={0} if rank == world - 1 else ())
        out.update(status=st, elapsed=time.monotonic() - t0)
        return
    out.update(bad=bad, statuses=statuses, calls=call, state=lar.state)


def main():
    scen = sys.argv[1]
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=30))
    out = {"rank": rank}
    sets = 1 if scen == "oneset" else 2
    if scen.startswith("ll_"):
        fab = P.LineFabric(rank, world, max_tokens=48, max_n=256, directory=os.environ["PROTO_DIR"], tag=scen)
    else:
        fab = P.PeerFabric(rank, world, max_tokens=96, max_n=384, tile_t=32, directory=os.environ["PROTO_DIR"],
                           tag=f"{scen}", sets=sets)
    try:
        if scen.startswith("ll_"):
            run_lines(scen, fab, rank, world, out)
        elif scen == "exact":
            bad, statuses = [], []
            shapes = [(1, 64, 128), (5, 64, 256), (16, 128, 128), (33, 64, 384), (96, 32, 256), (47, 64, 128)]
            call = 0
            for cs in (1, 2, 3):
                ar = P.EmulatedAllReduce(fab, tile_t=32, cs=cs, grid=7)
                for T, K, N in shapes:
                    x, w = inputs(rank, call, T, K, N)
                    y, st = ar(x, w, seed=rank * 7919 + call)
                    parts, fp32 = expected(world, call, T, K, N)
                    ref = P.reduce_rank_order(parts)
                    yb = y.view(torch.int16).numpy().view(np.uint16)
                    if not np.array_equal(yb, ref):
                        bad.append([cs, T, N, "bits"])
                    err = (y.float() - fp32).abs().max().item() / max(1e-6, fp32.abs().max().item())
                    if err > 2e-2:
                        bad.append([cs, T, N, f"err {err:.3g}"])
                    statuses.append(st)
                    call += 1
            out.update(bad=bad, statuses=statuses, calls=call)
        elif scen in ("skew", "oneset"):
            ar = P.EmulatedAllReduce(fab, tile_t=32, cs=1, grid=5, budget_s=1.5)
            wrong, statuses = 0, []
            for call in range(4):
                T, K, N = 40, 64, 256
                x, w = inputs(rank, call, T, K, N)
                y, st = ar(x, w, seed=call, stall_s=0.4 if rank == world - 1 else 0.0)
                parts, _ = expected(world, call, T, K, N)
                wrong += int(not np.array_equal(y.view(torch.int16).numpy().view(np.uint16),
                                                P.reduce_rank_order(parts)))
                statuses.append(st)
            out.update(wrong=wrong, statuses=statuses)
        elif scen == "drop":
            ar = P.EmulatedAllReduce(fab, tile_t=32, cs=2, grid=3, budget_s=0.5)
            x, w = inputs(rank, 0, 40, 64, 128)
            import time
            t0 = time.monotonic()
            _, st = ar(x, w, drop={(0, 0)} if rank == world - 1 else ())
            out.update(status=st, elapsed=time.monotonic() - t0)
        print("PROTOJSON " + json.dumps(out), flush=True)
    finally:
        fab.close()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
