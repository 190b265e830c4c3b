"""gloo rank for the failure-detection tests. Scenario from argv[1]:

  crash     -- rank world-1 raises after 2 steps; the others must detect it
  leave     -- rank world-1 leaves gracefully after 2 steps
  dropflag  -- rank 1 never publishes the flag rank 0 waits for
  collective -- rank 1 skips one all_reduce; rank 0's must time out

Prints one "FAULTJSON {...}" line per surviving rank."""
import faulthandler
import json
import os
import sys
import time
import datetime

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))))

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

from sched_pass_b200.parallel.health import (Heartbeat, RankFailure, guarded, publish_flag,  # noqa: E402
                                             wait_flag)


faulthandler.enable()  # a native crash prints the Python stack of every thread


def main():
    scenario = sys.argv[1]
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=4))
    hb = Heartbeat(rank, world, interval=0.1, timeout=1.0).start()
    out = {"rank": rank, "scenario": scenario}
    t0 = time.monotonic()
    x = torch.ones(4)
    try:
        if scenario in ("crash", "leave"):
            victim = world - 1
            for step in range(200):
                if rank == victim and step == 2:
                    if scenario == "crash":
                        os._exit(3)  # dies without any goodbye
                    hb.leave()
                    out["left"] = True
                    break
                guarded(hb, dist.all_reduce, x)
                time.sleep(0.02)
        elif scenario == "dropflag":
            store = hb.store
            if rank == 0:
                out["got"] = wait_flag(store, "step0", budget_s=0.5)
                publish_flag(store, "done")
                wait_flag(store, "ack", budget_s=5.0)  # the store lives in rank 0: outlive the peer's reads
            else:
                # "forgets" step0; still proves it is alive and waits for rank 0
                out["got"] = wait_flag(store, "done", budget_s=5.0)
                publish_flag(store, "ack")
        elif scenario == "collective":
            if rank != 1:
                dist.all_reduce(x)
        out["ok"] = True
    except RankFailure as e:
        out["failure"] = e.ranks
    except RuntimeError as e:
        out["error"] = str(e)[:200]
    out["elapsed"] = round(time.monotonic() - t0, 3)
    hb.stop()
    print("FAULTJSON " + json.dumps(out), flush=True)
    os._exit(0)  # no collective teardown with a peer that may be gone


if __name__ == "__main__":
    main()
