"""One gloo rank of the sequence-parallel protocol emulation
(sched_pass_b200/parallel/sp_protocol.py). Scenario from argv[1]; prints one
``SPJSON {...}`` line."""
import faulthandler
import datetime
import json
import os
import sys
import time

import numpy as np
import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))))
from sched_pass_b200.parallel import protocol as P  # noqa: E402
from sched_pass_b200.parallel import sp_protocol as S  # noqa: E402

H, K, EPS = 256, 64, 1e-5


def inputs(rank, call, T):
    g = torch.Generator().manual_seed(1000 * call + rank)
    x = torch.randn(T, K, generator=g).to(torch.bfloat16)
    w = (torch.randn(H, K, generator=g) / K ** 0.5).to(torch.bfloat16)
    return x, w


def norm_weight(call):
    g = torch.Generator().manual_seed(77 + call)
    return P.to_bf16_bits(1.0 + 0.1 * torch.randn(H, generator=g))


faulthandler.enable()  # a native crash prints the Python stack of every thread


def main():
    scen = sys.argv[1]
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=30))
    fab = S.SpFabric(rank, world, max_tokens=64, hidden=H, directory=os.environ["PROTO_DIR"], tag=scen)
    out = {"rank": rank}
    try:
        if scen in ("exact", "skew"):
            sp = S.EmulatedSequenceParallel(fab, budget_s=2.0)
            # token counts shrink and grow again: stale flags from a larger
            # call must not release rows of a smaller or later one
            Ts = [48, 5, 1, 33, 64, 7, 48]
            g0 = torch.Generator().manual_seed(5)
            res_full = P.to_bf16_bits(torch.randn(64, H, generator=g0))  # same on every rank
            bad, statuses = [], []
            for call, T in enumerate(Ts):
                x, w = inputs(rank, call, T)
                sp.linear_rs(x, w, seed=rank * 31 + call)
                res = res_full[:T].copy()
                wn = norm_weight(call)
                stall = 0.3 if (scen == "skew" and rank == world - 1) else 0.0
                g, delta, st = sp.reduce_norm(res, wn, EPS, seed=call, stall_s=stall)
                got, st2 = sp.consume(g, T)
                statuses += [st, st2]
                parts = np.stack([P.to_bf16_bits(a.float() @ b.float().t())
                                  for a, b in (inputs(r, call, T) for r in range(world))])
                want_delta = P.reduce_rank_order(parts)
                lo, hi = S.owned_rows(rank, world, T)
                if not np.array_equal(delta, want_delta[lo:hi]):
                    bad.append([call, "delta bits"])
                want_res = P.to_bf16_bits(torch.from_numpy(P.from_bf16_bits(want_delta)
                                                           + P.from_bf16_bits(res_full[:T])))
                if not np.array_equal(res[lo:hi], want_res[lo:hi]):
                    bad.append([call, "residual bits"])
                want = S.rmsnorm_bf16(want_res, wn, EPS)
                if not np.array_equal(got, want):
                    bad.append([call, "gathered rows"])
                # every rank reads the same gathered rows
                allg = [None] * world
                dist.all_gather_object(allg, got.tobytes())
                if any(a != allg[0] for a in allg):
                    bad.append([call, "ranks disagree"])
            out.update(bad=bad, statuses=statuses)
        elif scen == "drop":
            sp = S.EmulatedSequenceParallel(fab, budget_s=0.5)
            x, w = inputs(rank, 0, 24)
            t0 = time.monotonic()
            # the last rank loses its push of row 0, n-tile 1
            sp.linear_rs(x, w, drop={(0, 1)} if rank == world - 1 else ())
            res = np.zeros((24, H), dtype=np.uint16)
            g, _, st = sp.reduce_norm(res, norm_weight(0), EPS)
            _, st2 = sp.consume(g, 24)
            out.update(status=st, consume=st2, elapsed=time.monotonic() - t0)
        print("SPJSON " + json.dumps(out), flush=True)
    finally:
        fab.close()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
