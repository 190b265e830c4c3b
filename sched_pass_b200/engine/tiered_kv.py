"""Tiered KV store: the device page pool spills to pinned host memory.

Pages live in one of three places:

* device pages ``[0, n_device)`` -- handed out by the scheduler's allocator;
* host pages, named ``HOST_BASE + h`` in a request's page list -- a pinned
  host pool with the device pool's layout ([layers, pages, heads, 16, 128]);
* staging pages ``[n_device, n_device + n_staging)`` of the device pool --
  never owned by a request: each step copies the host pages that step reads
  into them, and the step's block table points there.

Spilling happens when the allocator runs dry (the scheduler calls ``spill``
before it would preempt anyone). Victims are chosen by the scheduling
plane's own signals, in this order:

1. pages a request will never read again: beyond its shed horizon
   (``tau`` tokens) -- moving them costs one copy and never comes back;
2. pages of the least urgent decode requests (``urgency``, the plane's q),
   oldest first.

A request's last page (where the next token's K/V is appended) and requests
still in prefill are never spilled. Each step, ``stage`` gathers the host
pages inside every decode request's read horizon into staging pages, in the
order the decode kernel will claim their tasks (most urgent request first,
the order pi and the policy rows favour), and launches one copy kernel over
PCIe on the engine's stream, so the step's kernels run after it.

The copies are ``csrc/kernels/kv_tier.cu`` (zero-copy loads/stores of the
mapped pinned pool). The reference names KV tiering as its unbuilt "MOVE"
lever (ROADMAP.md:462-482 of jc-su/sched-pass); this is the mechanism.
"""
from __future__ import annotations

import math

import numpy as np
import torch

from .._ext import ext

HOST_BASE = 1 << 30


def is_host(page: int) -> bool:
    return page >= HOST_BASE


class TieredKV:
    def __init__(self, kv, n_device: int, n_staging: int, n_host: int, device):
        self.kv = kv
        self.n_device = int(n_device)
        self.n_staging = int(n_staging)
        self.n_host = int(n_host)
        self.device = torch.device(device)
        if kv.num_pages < self.n_device + self.n_staging:
            raise ValueError("the device KV pool must hold the allocator's pages plus the staging pages")
        L, _, H, P, D = kv.k.shape
        shape = (L, self.n_host, H, P, D)
        pin = self.device.type == "cuda"
        self.host_k = torch.zeros(shape, dtype=kv.k.dtype, pin_memory=pin)
        self.host_v = torch.zeros(shape, dtype=kv.v.dtype, pin_memory=pin)
        self._free_host = list(range(self.n_host - 1, -1, -1))
        self.spilled_pages = 0
        self.staged_pages = 0
        self.last_stage = 0
        self._pairs_dev = torch.zeros(max(1, self.n_staging) * 2, dtype=torch.int32, device=self.device)
        self._pairs_host = torch.zeros(max(1, self.n_staging) * 2, dtype=torch.int32, pin_memory=pin)
        self._translation: dict = {}

    # ------------------------------------------------------------ host pool
    @property
    def host_free(self) -> int:
        return len(self._free_host)

    def free_host(self, pages) -> None:
        for p in pages:
            h = int(p) - HOST_BASE
            if not 0 <= h < self.n_host:
                raise ValueError(f"page {p} is not a host page")
            self._free_host.append(h)

    # ------------------------------------------------------------ spilling
    @staticmethod
    def horizon_pages(req) -> int:
        """Pages the decode kernel reads for this request (tau shortens it)."""
        n = req.total_len
        if req.tau and req.tau > 0:
            n = min(n, int(req.tau))
        return int(math.ceil(n / 16))

    def _victims(self, running, protect, want: int):
        from .request import State
        dec = [r for r in running if r.state == State.DECODE and r is not protect]
        out = []
        # 1. never read again: beyond the shed horizon, least urgent first
        for r in sorted(dec, key=lambda r: r.urgency):
            hz = self.horizon_pages(r)
            for i in range(hz, len(r.pages) - 1):
                if not is_host(r.pages[i]):
                    out.append((r, i))
                    if len(out) >= want:
                        return out
        # 2. read every step: least urgent requests, oldest pages first
        for r in sorted(dec, key=lambda r: r.urgency):
            for i in range(0, min(self.horizon_pages(r), len(r.pages) - 1)):
                if not is_host(r.pages[i]):
                    out.append((r, i))
                    if len(out) >= want:
                        return out
        return out

    def spill(self, want: int, running, protect=None) -> list:
        """Move up to ``want`` device pages to the host pool; returns the
        freed device page ids (the caller gives them back to its allocator).
        The copy is stream-ordered before any later reuse of those pages."""
        want = min(int(want), self.host_free)
        if want <= 0:
            return []
        victims = self._victims(running, protect, want)
        if not victims:
            return []
        freed, pairs = [], []
        for r, i in victims:
            h = self._free_host.pop()
            d = int(r.pages[i])
            pairs.append((d, h))
            r.pages[i] = HOST_BASE + h
            freed.append(d)
        self._copy(self.kv.k, self.kv.v, self.host_k, self.host_v, pairs)
        self.spilled_pages += len(pairs)
        return freed

    # ------------------------------------------------------------ staging
    def stage(self, decode_requests) -> None:
        """Copy the host pages each decode request reads this step into
        staging pages; ``pages_for`` then gives the translated page list."""
        self._translation.clear()
        pairs = []
        nxt = self.n_device
        for r in sorted(decode_requests, key=lambda r: -r.urgency):  # most urgent first
            if not any(is_host(p) for p in r.pages):
                continue
            hz = self.horizon_pages(r)
            tr = list(r.pages)
            for i, p in enumerate(r.pages):
                if not is_host(p):
                    continue
                if i >= hz:
                    tr[i] = 0  # never read this step: any valid device page
                    continue
                if nxt >= self.n_device + self.n_staging:
                    raise RuntimeError(
                        f"this step reads more host-resident KV pages than the {self.n_staging} staging "
                        "pages hold; raise kv_staging_pages (or spill less)")
                pairs.append((int(p) - HOST_BASE, nxt))
                tr[i] = nxt
                nxt += 1
            self._translation[id(r)] = tr
        self.last_stage = len(pairs)
        if pairs:
            self._copy(self.host_k, self.host_v, self.kv.k, self.kv.v, pairs)
            self.staged_pages += len(pairs)

    def pages_for(self, req):
        return self._translation.get(id(req), req.pages)

    # ------------------------------------------------------------ copies
    def _copy(self, src_k, src_v, dst_k, dst_v, pairs) -> None:
        n = len(pairs)
        if n == 0:
            return
        arr = np.asarray(pairs, dtype=np.int32).reshape(-1)
        if n * 2 > self._pairs_host.numel():
            self._pairs_host = torch.zeros(n * 2, dtype=torch.int32, pin_memory=self._pairs_host.is_pinned())
            self._pairs_dev = torch.zeros(n * 2, dtype=torch.int32, device=self.device)
        self._pairs_host[: n * 2].numpy()[:] = arr
        self._pairs_dev[: n * 2].copy_(self._pairs_host[: n * 2], non_blocking=True)
        ext().kv_page_copy(src_k, src_v, dst_k, dst_v, self._pairs_dev, n)
        # the pinned staging of the pairs is rewritten by the next call: keep
        # the host from getting ahead of the copy that reads it
        torch.cuda.current_stream(self.device).synchronize()
