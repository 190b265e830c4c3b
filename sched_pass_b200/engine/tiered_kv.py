"""Tiered KV store: the device page pool spills to pinned host memory, and
the spilled pages a step reads stream back one layer at a time.

Pages live in one of two pools:

* device pages ``[0, n_device)`` -- handed out by the scheduler's allocator;
* host pages, named ``HOST_BASE + h`` in a request's page list -- a pinned
  host pool with the device pool's layout ([layers, pages, heads, 16, 128]).

Spilling happens when the allocator runs dry (the scheduler calls ``spill``
before it would preempt anyone). Victims are chosen by the scheduling
plane's own signals, in this order:

1. pages a request will never read again: beyond its shed horizon
   (``tau`` tokens) -- moving them costs one copy and never comes back;
2. pages of the least urgent decode requests (``urgency``, the plane's q),
   oldest first.

A request's last page (where the next token's K/V is appended) and requests
still in prefill are never spilled.

Each step, ``stage`` gives every host page inside a decode request's read
horizon a staging slot ``s`` and writes ``split + s`` into the step's block
table (``split`` = the device pool's page count; the decode kernel reads
ids >= split from a second, staging pool). Slots are assigned in the order
the decode kernel claims its tasks (most urgent request first). The staging
pool holds ONE layer: two buffers alternate between even and odd layers, so
layer l's pages are copied over PCIe on a side stream while layer l-1
computes -- by the copy engines (one ``cudaMemcpyAsync`` per run of
consecutive host pages; spills take host pages in ascending order, so runs
are long) or by the zero-copy page-copy kernel (``csrc/kernels/kv_tier.cu``),
and the copy for layer l+2 waits until layer l's attention has read the
buffer. Staging costs 2 x slots x one layer's page of device memory, so the
read set of a step may exceed HBM (the 70B / 131k-context configuration).

With ``host_dtype="fp8"`` the host pool stores e4m3 pages with one fp32
scale per (layer, page, head, K|V): a spill quantizes, the staging copy
dequantizes back to bf16, so half the bytes cross PCIe per step (the
decode kernel still reads bf16). Cold pages then carry fp8 precision.

The reference names KV tiering as its unbuilt "MOVE" lever
(ROADMAP.md:462-482 of jc-su/sched-pass); this is the mechanism.
"""
from __future__ import annotations

import math

import numpy as np
import torch

from .. import ops
from .._ext import ext

HOST_BASE = 1 << 30


def is_host(page: int) -> bool:
    return page >= HOST_BASE


def coalesce_runs(pairs) -> list:
    """(host page, staging slot) pairs -> runs (first host page, first slot,
    length) over which both advance by one: each run is one contiguous copy
    per layer for K and one for V."""
    runs = []
    for h, s in pairs:
        if runs and runs[-1][0] + runs[-1][2] == h and runs[-1][1] + runs[-1][2] == s:
            runs[-1][2] += 1
        else:
            runs.append([h, s, 1])
    return [tuple(r) for r in runs]


class TieredKV:
    def __init__(self, kv, n_device: int, n_staging: int, n_host: int, device, host_dtype: str = "bf16",
                 stage_mode: str = "copy"):
        if host_dtype not in ("bf16", "fp8"):
            raise ValueError(f"host_dtype must be 'bf16' or 'fp8', not {host_dtype!r}")
        if stage_mode not in ("copy", "kernel"):
            raise ValueError(f"stage_mode must be 'copy' or 'kernel', not {stage_mode!r}")
        self.host_dtype = host_dtype
        # "copy": the copy engines move each layer's staged pages with one
        # cudaMemcpyAsync per run of consecutive host pages (K and V), on the
        # side stream, leaving the SMs to the overlapped layer; "kernel": the
        # zero-copy page-copy kernel (always used for the fp8 tier, which
        # dequantizes on the way)
        self.stage_mode = "kernel" if host_dtype == "fp8" else stage_mode
        self._runs: list = []
        self.kv = kv
        self.n_device = int(n_device)
        self.n_staging = max(1, int(n_staging))
        self.n_host = int(n_host)
        self.device = torch.device(device)
        if kv.num_pages < self.n_device:
            raise ValueError("the device KV pool is smaller than the allocator's page count")
        self.split = kv.num_pages  # block-table ids >= split name staging slots
        L, _, H, P, D = kv.k.shape
        self.layers = L
        on_cuda = self.device.type == "cuda"
        hdt = torch.uint8 if host_dtype == "fp8" else kv.k.dtype  # fp8 e4m3 bytes
        self.host_k = torch.zeros((L, self.n_host, H, P, D), dtype=hdt, pin_memory=on_cuda)
        self.host_v = torch.zeros((L, self.n_host, H, P, D), dtype=hdt, pin_memory=on_cuda)
        if host_dtype == "fp8":
            self.host_scale_k = torch.ones((L, self.n_host, H), dtype=torch.float32, pin_memory=on_cuda)
            self.host_scale_v = torch.ones((L, self.n_host, H), dtype=torch.float32, pin_memory=on_cuda)
        # two one-layer staging buffers (even / odd layers)
        self.stage_k = torch.zeros((2, self.n_staging, H, P, D), dtype=kv.k.dtype, device=self.device)
        self.stage_v = torch.zeros_like(self.stage_k)
        self._free_host = list(range(self.n_host - 1, -1, -1))
        self.spilled_pages = 0
        self.staged_pages = 0
        self.last_stage = 0
        cap = 2 * self.n_staging
        self.pairs_dev = torch.zeros(cap, dtype=torch.int32, device=self.device)  # (host page, slot)
        self.count_dev = torch.zeros(1, dtype=torch.int32, device=self.device)
        # two pinned sources of the page-pair upload, alternating per step: a
        # buffer is rewritten only after its copy of two steps ago has run
        # (its event), so staging never waits for the step in flight
        self._pairs_pin = [torch.zeros(cap + 1, dtype=torch.int32, pin_memory=on_cuda) for _ in range(2)]
        self._pin_done = [None, None]
        self._pin_k = 0
        self._spill_dev = torch.zeros(2, dtype=torch.int32, device=self.device)
        self._translation: dict = {}
        self._stream = torch.cuda.Stream(self.device) if on_cuda else None
        self._ev_fetch = [torch.cuda.Event() for _ in range(2)] if on_cuda else None
        self._ev_read = [torch.cuda.Event() for _ in range(2)] if on_cuda else None

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
            r.spilled_pages += 1
            freed.append(d)
        self._copy_all_layers(self.kv.k, self.kv.v, self.host_k, self.host_v, pairs)
        self.spilled_pages += len(pairs)
        return freed

    def _copy_all_layers(self, src_k, src_v, dst_k, dst_v, pairs) -> None:
        n = len(pairs)
        arr = torch.from_numpy(np.asarray(pairs, dtype=np.int32).reshape(-1))
        if n * 2 > self._spill_dev.numel():
            self._spill_dev = torch.zeros(n * 2, dtype=torch.int32, device=self.device)
        self._spill_dev[: n * 2].copy_(arr)  # pageable source: a synchronous copy
        if self.host_dtype == "fp8":
            ext().kv_page_copy_fp8(src_k, src_v, dst_k, dst_v, self.host_scale_k, self.host_scale_v, True,
                                   self._spill_dev, n, None, ops.status_buffer(self.device))
        else:
            ext().kv_page_copy(src_k, src_v, dst_k, dst_v, self._spill_dev, n, None, ops.status_buffer(self.device))

    # ------------------------------------------------------------ staging
    def stage(self, decode_requests) -> None:
        """Give each host page a decode request reads this step a staging
        slot (most urgent request first) and publish the pairs for the
        per-layer copies; ``pages_for`` gives the translated page list."""
        self._translation.clear()
        pairs = []
        for r in sorted(decode_requests, key=lambda r: -r.urgency):
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
                if len(pairs) >= self.n_staging:
                    raise RuntimeError(
                        f"this step reads more host-resident KV pages than the {self.n_staging} staging "
                        "slots hold; raise kv_staging_pages (or spill less)")
                tr[i] = self.split + len(pairs)
                pairs.append((int(p) - HOST_BASE, len(pairs)))
            self._translation[id(r)] = tr
        n = len(pairs)
        self.last_stage = n
        self.staged_pages += n
        self._runs = coalesce_runs(pairs)
        k = self._pin_k
        self._pin_k ^= 1
        pin = self._pairs_pin[k]
        if self._pin_done[k] is not None:
            self._pin_done[k].synchronize()  # this buffer's upload of two steps ago has run
        buf = pin.numpy()
        buf[0] = n
        if n:
            buf[1:1 + 2 * n] = np.asarray(pairs, dtype=np.int32).reshape(-1)
        self.count_dev.copy_(pin[:1], non_blocking=True)
        if n:
            self.pairs_dev[: 2 * n].copy_(pin[1:1 + 2 * n], non_blocking=True)
        if self.device.type == "cuda":
            ev = torch.cuda.Event()
            ev.record(torch.cuda.current_stream(self.device))
            self._pin_done[k] = ev

    def pages_for(self, req):
        return self._translation.get(id(req), req.pages)

    # ------------------------------------------------------------ per-layer streaming
    def _fetch(self, layer: int) -> None:
        b = layer & 1
        if self.stage_mode == "copy":
            for h0, s0, n in self._runs:  # pinned -> device: cudaMemcpyAsync on the current (side) stream
                self.stage_k[b, s0:s0 + n].copy_(self.host_k[layer, h0:h0 + n], non_blocking=True)
                self.stage_v[b, s0:s0 + n].copy_(self.host_v[layer, h0:h0 + n], non_blocking=True)
            return
        if self.host_dtype == "fp8":
            ext().kv_page_copy_fp8(self.host_k[layer:layer + 1], self.host_v[layer:layer + 1],
                                   self.stage_k[b:b + 1], self.stage_v[b:b + 1],
                                   self.host_scale_k[layer:layer + 1], self.host_scale_v[layer:layer + 1], False,
                                   self.pairs_dev, self.n_staging, self.count_dev, ops.status_buffer(self.device))
            return
        ext().kv_page_copy(self.host_k[layer:layer + 1], self.host_v[layer:layer + 1],
                           self.stage_k[b:b + 1], self.stage_v[b:b + 1], self.pairs_dev, self.n_staging,
                           self.count_dev, ops.status_buffer(self.device))

    def begin_forward(self) -> None:
        """Fork the copy stream and start the copies of layers 0 and 1."""
        main = torch.cuda.current_stream(self.device)
        self._stream.wait_stream(main)
        with torch.cuda.stream(self._stream):
            for layer in range(min(2, self.layers)):
                self._fetch(layer)
                self._ev_fetch[layer & 1].record(self._stream)

    def before_attention(self, layer: int):
        """Wait for this layer's pages; returns the decode kernel's staging pool."""
        b = layer & 1
        torch.cuda.current_stream(self.device).wait_event(self._ev_fetch[b])
        return (self.stage_k[b], self.stage_v[b], self.split)

    def after_attention(self, layer: int) -> None:
        """Layer ``layer`` has read its buffer: refill it for ``layer + 2``."""
        b = layer & 1
        nxt = layer + 2
        if nxt >= self.layers:
            return
        self._ev_read[b].record(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(self._stream):
            self._stream.wait_event(self._ev_read[b])
            self._fetch(nxt)
            self._ev_fetch[b].record(self._stream)

    def end_forward(self) -> None:
        torch.cuda.current_stream(self.device).wait_stream(self._stream)
