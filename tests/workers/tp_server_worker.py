"""One gloo rank of the tensor-parallel server test: rank 0 runs
TPEngineServer and submits requests, the other ranks follow; every rank has
a fake engine behind the real scheduler. Prints one ``SRVJSON {...}`` line."""
import faulthandler
import datetime
import json
import os
import sys

import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))))
from sched_pass_b200.engine.scheduler import Scheduler  # noqa: E402
from sched_pass_b200.engine.server import TPEngineServer, follow  # noqa: E402


class FakeEngine:
    """Scheduler + a model that emits (previous token + 1) mod vocab; each
    step advances the clock by 1 ms. Records every finished request."""

    def __init__(self):
        self.sched = Scheduler(4096, 16, 8, 64, 4096)
        self.clock = 0.0
        self.device = None
        self.finished = {}
        self.steps = 0

    def add_request(self, r):
        self.sched.add(r)

    def abort(self, r):
        return self.sched.abort(r)

    def has_work(self):
        return not self.sched.idle

    def step(self):
        plan = self.sched.schedule()
        sampled = {r.rid: (r.next_input_token() + 1) % 1000 for r in plan.decode}
        for r, start, n in plan.prefill:
            if start + n >= r.prompt_len:
                sampled[r.rid] = (int(r.prompt[-1]) + 1) % 1000
        self.clock += 0.001
        done = self.sched.commit(plan, sampled, self.clock)
        for r in done:
            self.finished[r.rid] = list(r.output)
        self.steps += 1
        return plan, done


def leave_scenario(rank, eng, out):
    """The last rank follows a few rounds, then leaves between rounds: rank
    0's server must fail its pending requests instead of hanging."""
    import time

    from sched_pass_b200.parallel.health import Heartbeat
    world = dist.get_world_size()
    hb = Heartbeat(rank, world, interval=0.05, timeout=1.0).start()
    dist.barrier()
    if rank == 0:
        srv = TPEngineServer(eng, heartbeat=hb, idle_wait_s=0.01).start()
        futs = [srv.submit(list(range(20)), 4000) for _ in range(4)]  # never finish before the failure
        t0 = time.monotonic()
        errs = []
        for f in futs:
            try:
                f.result(timeout=60)
                errs.append(None)
            except Exception as e:  # noqa: BLE001
                errs.append(type(e).__name__)
        out.update(failed=errs, elapsed=time.monotonic() - t0, error=repr(srv.error))
        srv._stop.set()
    elif rank == world - 1:
        follow(eng, heartbeat=hb, max_rounds=20)
        hb.leave()
        out["left"] = True
    else:
        try:
            follow(eng, heartbeat=hb)
            out["follower"] = "stopped"
        except Exception as e:  # noqa: BLE001
            out["follower"] = type(e).__name__
    print("SRVJSON " + json.dumps(out), flush=True)
    os._exit(0)  # skip the group teardown: a peer is gone


faulthandler.enable()  # a native crash prints the Python stack of every thread


def main():
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=60 if len(sys.argv) < 2 else 5))
    rank = dist.get_rank()
    eng = FakeEngine()
    out = {"rank": rank}
    if len(sys.argv) > 1 and sys.argv[1] == "leave":
        return leave_scenario(rank, eng, out)
    if rank == 0:
        srv = TPEngineServer(eng).start()
        futs = [srv.submit(list(range(5 + 7 * i)), 3 + i % 4) for i in range(12)]
        bad = srv.submit(list(range(5000)), 3)  # beyond max_context: fails on rank 0 only, never sent
        long = srv.submit(list(range(9)), 3500, name="long")  # cancelled while running
        res = [f.result(timeout=60) for f in futs]
        out["bad_rejected"] = bad.exception(timeout=60) is not None
        srv.cancel("long")
        import concurrent.futures as cf
        try:
            long.result(timeout=60)
            out["long_cancelled"] = False
        except cf.CancelledError:
            out["long_cancelled"] = True
        srv.stop()
        out["outputs"] = {str(i): r["output_ids"] for i, r in enumerate(res)}
        out["error"] = repr(srv.error) if srv.error else None
    else:
        follow(eng)
    out["steps"] = eng.steps
    out["idle"] = eng.sched.idle and eng.sched.alloc.free == eng.sched.alloc.num_pages
    out["finished"] = {str(k): v for k, v in sorted(eng.finished.items())}
    print("SRVJSON " + json.dumps(out), flush=True)
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
