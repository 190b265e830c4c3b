"""Host-side failure detection for multi-rank runs.

The device side never waits without a bound: every spin on a peer flag, an
mbarrier or a cluster-launch-control response in this framework's kernels
gives up after a wall-clock budget and writes a status code the host reads
(``ops.check_status``). This module is the host side:

* ``Heartbeat`` -- each rank publishes a sequence number in the
  torch.distributed store from a background thread; every rank can ask which
  peers have gone silent (``dead_ranks``) or left (``leave``) and raise
  ``RankFailure`` before its next collective or fused-collective launch
  (``check``), so survivors stop between steps instead of entering a kernel
  that would wait for a rank that is gone. Staleness is judged on the
  observer's own clock (a sequence that stopped changing), so clock skew
  between hosts does not matter.
* ``publish_flag`` / ``wait_flag`` -- a store-backed flag with a bounded wait
  (the host-side image of the kernels' peer flags), used to emulate and test
  lost messages.
* ``guarded`` -- runs one step's collective work after a health check and
  turns a collective timeout into ``RankFailure``.

Process groups should be created with a short timeout
(``parallel.tp.init_distributed(timeout_s=...)``) so that a collective with
a missing peer ends with an error.
"""
from __future__ import annotations

import threading
import time


class RankFailure(RuntimeError):
    def __init__(self, ranks, why: str):
        self.ranks = sorted(set(int(r) for r in ranks))
        super().__init__(f"rank(s) {self.ranks} failed: {why}")


def default_store():
    import torch.distributed as dist
    from torch.distributed import distributed_c10d as c10d
    if not dist.is_initialized():
        raise RuntimeError("torch.distributed is not initialised")
    return c10d._get_default_store()


class Heartbeat:
    """Liveness of every rank through the store (one key per rank)."""

    LEFT = b"left"

    def __init__(self, rank: int, world: int, store=None, interval: float = 0.25, timeout: float = 3.0,
                 prefix: str = "sched/hb"):
        self.rank, self.world = int(rank), int(world)
        self.store = store if store is not None else default_store()
        self.interval, self.timeout = float(interval), float(timeout)
        self.prefix = prefix
        self._seq = 0
        self._stop = threading.Event()
        self._thread: threading.Thread | None = None
        # observer state: last value seen per rank and when it last changed
        self._seen: dict[int, tuple[bytes, float]] = {}
        self._t0 = time.monotonic()

    def _key(self, r: int) -> str:
        return f"{self.prefix}/{r}"

    def beat(self) -> None:
        self._seq += 1
        self.store.set(self._key(self.rank), str(self._seq).encode())

    def _run(self) -> None:
        while not self._stop.wait(self.interval):
            try:
                self.beat()
            except Exception:  # noqa: BLE001 - the store went away: the job is ending
                return

    def start(self) -> "Heartbeat":
        self.beat()
        if self._thread is None:
            self._thread = threading.Thread(target=self._run, name=f"hb-{self.rank}", daemon=True)
            self._thread.start()
        return self

    def stop(self) -> None:
        self._stop.set()
        if self._thread is not None:
            self._thread.join(2 * self.interval + 1.0)
            self._thread = None

    def leave(self) -> None:
        """Graceful exit between steps: peers see this rank as gone at once."""
        self.stop()
        self.store.set(self._key(self.rank), self.LEFT)

    def _read(self, r: int):
        k = self._key(r)
        if not self.store.check([k]):
            return None
        return self.store.get(k)

    def dead_ranks(self) -> list:
        now = time.monotonic()
        dead = []
        for r in range(self.world):
            if r == self.rank:
                continue
            v = self._read(r)
            if v == self.LEFT:
                dead.append(r)
                continue
            prev = self._seen.get(r)
            if prev is None or prev[0] != v:
                self._seen[r] = (v, now)
                continue
            if now - prev[1] > self.timeout:
                dead.append(r)
        # a rank that never published counts as dead once the grace period ends
        if now - self._t0 > self.timeout:
            dead += [r for r in range(self.world) if r != self.rank and self._seen.get(r, (None,))[0] is None
                     and r not in dead]
        return sorted(dead)

    def check(self) -> None:
        dead = self.dead_ranks()
        if dead:
            raise RankFailure(dead, "no heartbeat")


def publish_flag(store, name: str, value: int = 1) -> None:
    store.set(f"sched/flag/{name}", str(int(value)).encode())


def wait_flag(store, name: str, value: int = 1, budget_s: float = 1.0, poll_s: float = 0.005) -> bool:
    """Bounded wait for a flag; False once the budget is spent (never hangs)."""
    key = f"sched/flag/{name}"
    t0 = time.monotonic()
    while True:
        if store.check([key]) and int(store.get(key)) >= value:
            return True
        if time.monotonic() - t0 > budget_s:
            return False
        time.sleep(poll_s)


def guarded(hb: Heartbeat, fn, *args, **kwargs):
    """Run one step's collective work: check peers first, and report a
    collective that timed out (a peer vanished mid-step) as RankFailure."""
    hb.check()
    try:
        return fn(*args, **kwargs)
    except RuntimeError as e:
        text = str(e).lower()
        if "timed out" in text or "timeout" in text or "connection" in text or "closed" in text:
            # the collective noticed first; give the heartbeat time to name the rank
            deadline = time.monotonic() + 2 * hb.timeout + hb.interval
            dead = hb.dead_ranks()
            while not dead and time.monotonic() < deadline:
                time.sleep(hb.interval)
                dead = hb.dead_ranks()
            raise RankFailure(dead or [-1], f"collective failed: {e}") from e
        raise
