"""One gloo rank of the MoE exchange emulation
(sched_pass_b200/parallel/ep_protocol.py). Scenario from argv[1], buffer
sets from argv[2]; prints one ``EPJSON {...}`` line."""
import datetime
import faulthandler
import json
import os
import sys

import numpy as np
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))))
from sched_pass_b200.parallel import ep_protocol as EP  # noqa: E402
from sched_pass_b200.parallel.protocol import STATUS_OK  # noqa: E402

faulthandler.enable()
E_LOCAL, K, H, T = 2, 2, 32, 8


def experts_all(world):
    g = np.random.default_rng(5)
    return (g.standard_normal((world * E_LOCAL, H, H)) / np.sqrt(H)).astype(np.float32)


def layer_inputs(rank, world, layer, avoid=None):
    g = np.random.default_rng(1000 * layer + rank)
    x = g.standard_normal((T, H)).astype(np.float32)
    E = world * E_LOCAL
    allowed = [e for e in range(E) if avoid is None or e // E_LOCAL != avoid]
    ids = np.stack([g.choice(allowed, size=K, replace=False) for _ in range(T)]).astype(np.int32)
    wts = g.random((T, K)).astype(np.float32)
    return x, ids, wts


def reference(x, ids, wts, kept, W):
    out = np.zeros((T, H), dtype=np.float32)
    for k in range(K):
        for t in range(T):
            if kept[t, k]:
                out[t] += (x[t] @ W[ids[t, k]].T) * np.float32(wts[t, k])
    return out


def main():
    scen, sets = sys.argv[1], int(sys.argv[2])
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=60))
    cap = 64 if scen != "ep_drops" else 3
    fab = EP.EpFabric(rank, world, E_LOCAL, cap, H, T, K, os.environ["PROTO_DIR"], f"{scen}{sets}", sets=sets)
    W = experts_all(world)
    mine = W[rank * E_LOCAL:(rank + 1) * E_LOCAL]
    ex = EP.EmulatedMoEExchange(fab, budget_s=1.0)
    out = {"rank": rank, "wrong": 0, "statuses": [], "dropped": 0}
    try:
        for layer in range(6 if scen != "ep_skew" else 4):
            avoid = world - 1 if (scen == "ep_skew" and rank == 0) else None
            x, ids, wts = layer_inputs(rank, world, layer, avoid)
            stall = 0.3 if (scen == "ep_skew" and rank == world - 1) else 0.0
            y, kept, st = ex(x, ids, wts, mine, stall_s=stall)
            out["wrong"] += int(not np.array_equal(y, reference(x, ids, wts, kept, W)))
            out["statuses"].append(st)
            out["dropped"] += int((~kept).sum())
    finally:
        print("EPJSON " + json.dumps(out), flush=True)
        fab.close()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
