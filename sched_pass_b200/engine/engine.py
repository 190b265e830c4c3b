"""The serving engine: scheduler -> step plan -> device buffers -> forward.

Per step:
  1. the scheduler picks the decode set and the prefill chunks;
  2. the planner (numpy + the native host runtime) lays out token rows
     (decode rows first), positions, KV slots, block-table rows, the decode
     work items (each request split into S KV chunks so that even small
     batches fill the SMs) and the prefill query tiles, all into ONE pinned
     int32 buffer that is copied to the device with one async copy;
  3. the scheduling levers are programmed: the controller orders the decode
     tasks (LPT / region order when cluster launch control is armed), the
     probe cadence switches the per-task timer on every ``timer_every`` steps,
     shed budgets are written for low-urgency requests, and the control
     block is published (stream-ordered, before the forward);
  4. decode-only steps replay a CUDA graph captured for the batch bucket;
     mixed steps run eagerly;
  5. the sampled token ids come back with one D2H copy; the timer of a probe
     step is folded into the controller's cost model.

Timing of a step is taken on the device (CUDA events around the forward).
"""
from __future__ import annotations

import math
import os
import time
import weakref
from collections import deque
from dataclasses import dataclass, field

import numpy as np
import torch

from .. import _ext, ops
from ..models.config import ModelConfig
from ..models.llama import ForwardBatch, KVCache, Llama, init_weights
from ..runtime.controller import SchedControlPlane
from ..runtime.sched_rt import SchedPlane
from . import native
from .plugin import HookRunner, SchedPlugin, SchedPluginConfig
from .request import Request, State
from .scheduler import Scheduler, StepPlan

DECODE_BUCKETS = (1, 2, 4, 8, 12, 16, 24, 32, 40, 48, 56, 64, 80, 96, 112, 128, 160, 192, 224, 256)
Q_TILE = 128  # query rows per prefill-attention tile (ops.PREFILL_TILE_ROWS)
MIXED_SEGMENTS = 4  # prefill requests per step of a fixed-shape (graph) mixed step


def order_prefill_tiles(tiles: list, mode: str = "lpt") -> list:
    """pi for prefill attention: the order of the query tiles in the launch
    (tile i runs as CTA column i, so the order is the order the hardware
    starts them). "lpt": longest first by causal work, rows x keys
    (nq x (q_pos0 + nq)), ties in plan order -- the reference's prefill pi
    (jc-su/sched-pass ROADMAP.md:450-451: -15.2 % at 48 requests). "identity":
    plan order. Each tile writes only its own rows, so every order gives
    the same bits. Tiles are (bt row, first q row, rows, first position)."""
    if mode == "identity" or len(tiles) < 2:
        return list(tiles)
    if mode != "lpt":
        raise ValueError(f"unknown prefill tile order {mode!r}")
    return sorted(tiles, key=lambda t: -(t[2] * (t[3] + t[2])))


@dataclass
class EngineConfig:
    max_batch: int = 256
    max_prefill_tokens: int = 4096
    max_step_tokens: int = 0        # cap on decode + prefill tokens per step (0 = none; see Scheduler)
    prefill_order: str = "lpt"      # order of prefill attention tiles: "lpt" (longest first) | "identity"
    prefix_cache: bool = False      # share the KV pages of common prompt prefixes (not with tiered KV)
    admission: str = "fcfs"         # waiting-queue order: fcfs | urgency | lpm (longest cached prefix)
    mixed_graphs: bool = True       # with max_step_tokens: pad mixed steps to a fixed shape per decode
                                    # bucket and replay them from CUDA graphs
    max_context: int = 4096
    num_pages: int = 0              # 0: sized from max_batch * max_context
    cuda_graphs: bool = True
    levers: bool = True             # weave the levers into the decode kernel
    acquire: str = "static"         # static | ticket | clc | auto
    timer_every: int = 8            # probe cadence of the per-task timer (0 = never)
    plan_every: int = 1             # re-order cadence
    lpt_block: int = 16
    clc_uncertainty: float = 0.75   # arm CLC above this estimator uncertainty (auto)
    shed_fraction: float = 0.0      # fraction of lowest-urgency requests given a tau
    shed_ratio: float = 0.5         # tau = ratio * context length
    target_tasks: int = 0           # decode tasks to aim for (0 = one per SM)
    seed: int = 0
    verbose: bool = False           # print the scheduling plugin's effective config
    host_kv_pages: int = 0          # tiered KV: pinned host pages the device pool spills to (0 = off)
    kv_staging_pages: int = 0       # staging slots (one layer of a host page each; 0 = host_kv_pages)
    host_kv_dtype: str = "bf16"     # host pool storage: "bf16" or "fp8" (e4m3 + per-head page scales)
    kv_stage_mode: str = "copy"     # tiered KV staging: "copy" (cudaMemcpyAsync runs on a side stream)
                                    # or "kernel" (zero-copy page-copy kernel; always for the fp8 tier)
    clock_sync: bool = True         # tensor parallel: advance every rank's workload clock by the slowest
                                    # rank's step time (one small collective per step); off when the
                                    # caller admits requests on a clock of its own


PENDING = -1  # placeholder of a sampled token the host has not read back yet


def _weak_call(obj, name: str):
    """A callable that calls ``obj.name(...)`` without keeping ``obj`` alive
    (None once ``obj`` is gone)."""
    ref = weakref.ref(obj)

    def call(*args):
        o = ref()
        return getattr(o, name)(*args) if o is not None else None
    return call


@dataclass
class _InFlight:
    plan: StepPlan
    info: dict
    ev0: object
    ev1: object
    done_ev: object
    buf: int
    pend: list       # (request, index in its output, row of the sampled ids)
    graph: bool
    finished: list   # requests whose last token this step produces


@dataclass
class StepStats:
    n_decode: int
    n_prefill_tokens: int
    device_ms: float
    graph: bool


def summarize_steps(stats: list) -> dict:
    """Aggregate of engine steps: counts by kind, device time (total, mean,
    p50/p99 of decode-only steps), the share of steps replayed from CUDA
    graphs, and decode / prefill tokens."""
    if not stats:
        return {"steps": 0}
    dec = sorted(s.device_ms for s in stats if s.n_prefill_tokens == 0)
    pct = lambda v, q: float(v[min(len(v) - 1, max(0, int(math.ceil(q * len(v))) - 1))]) if v else None  # noqa: E731
    total = sum(s.device_ms for s in stats)
    return {"steps": len(stats), "decode_only_steps": len(dec),
            "mixed_or_prefill_steps": len(stats) - len(dec),
            "graph_share": round(sum(1 for s in stats if s.graph) / len(stats), 4),
            "device_ms_total": round(total, 3), "device_ms_mean": round(total / len(stats), 4),
            "decode_step_ms_p50": pct(dec, 0.5), "decode_step_ms_p99": pct(dec, 0.99),
            "decode_tokens": sum(s.n_decode for s in stats),
            "prefill_tokens": sum(s.n_prefill_tokens for s in stats),
            # decode tokens per second of device time of these steps (this GPU, or the box under TP)
            "decode_tok_s_device": round(sum(s.n_decode for s in stats) / (total / 1e3), 1) if total > 0 else None}


class Engine:
    """Single-process engine for one tensor-parallel rank (``tp`` from
    ``parallel.tp``; None for one GPU). Every rank of a TP group runs the same
    scheduler on the same requests, so plans agree without communication."""

    def __init__(self, cfg: ModelConfig, ecfg: EngineConfig | None = None, device="cuda", tp=None,
                 weights=None, model_factory=None):
        self.cfg = cfg
        self.ecfg = ecfg or EngineConfig()
        e = self.ecfg
        self.device = torch.device(device)
        self.tp = tp
        tp_size = tp.world if tp is not None else 1
        tp_rank = tp.rank if tp is not None else 0
        self.max_pages_per_req = (e.max_context + 15) // 16
        if not e.num_pages:
            e.num_pages = e.max_batch * self.max_pages_per_req + 64
        self.kv = KVCache(cfg, e.num_pages, self.device, tp_size=tp_size)
        self.tier = None
        if e.host_kv_pages:
            from .tiered_kv import TieredKV
            self.tier = TieredKV(self.kv, e.num_pages, e.kv_staging_pages or e.host_kv_pages,
                                 e.host_kv_pages, self.device, host_dtype=e.host_kv_dtype,
                                 stage_mode=e.kv_stage_mode)
        if weights is None:
            weights = init_weights(cfg, self.device, tp_rank, tp_size, seed=e.seed,
                                   moe_builder=getattr(model_factory, "moe_builder", None))
        T = max(e.max_prefill_tokens + e.max_batch, 256)
        if model_factory is not None:
            self.model = model_factory(cfg, weights, self.kv, self.device, tp, T, e.max_context + 16)
        else:
            self.model = Llama(cfg, weights, self.kv, self.device, tp=tp, max_tokens=T,
                               max_pos=e.max_context + 16)
        self.sched = self.new_scheduler(tier=self.tier)
        self.hkv = cfg.n_kv_heads // tp_size
        self.sms = torch.cuda.get_device_properties(self.device).multi_processor_count
        self.target_tasks = e.target_tasks or self.sms
        self._alloc_buffers(T)
        # scheduling control plane (device-resident tables)
        max_tasks = e.max_batch * 8 * self.hkv
        self.plane = SchedPlane(max_tasks=max_tasks, device=str(self.device), mode="device")
        self.controller = SchedControlPlane(policy="lpt")
        self.R = self._resident_prefix()
        self.step_no = 0
        self.graphs: dict[int, tuple] = {}  # key -> (graph, splits, items, kernel launches it holds)
        self.graph_launches = 0  # kernel launches replayed from graphs (the extension counts the rest)
        self._inflight: deque = deque()  # steps enqueued whose tokens the host has not read yet
        # through a weak reference: the scheduler must not keep the engine (and
        # its CUDA graphs, which may hold collectives) alive after its owner drops it
        self.sched.before_preempt = _weak_call(self, "_before_preempt")
        self._pool = None
        self.stats: list[StepStats] = []
        self.clock = 0.0  # workload clock in seconds (device time + idle gaps)
        # per-step hooks; the scheduling plugin programs the levers
        self.hooks = HookRunner()
        self.plugin = None
        if e.levers:
            pcfg = SchedPluginConfig.from_engine_config(e).with_env()
            self.plugin = SchedPlugin(pcfg).register(self) if e.verbose else SchedPlugin(pcfg)
            if not e.verbose:
                self.hooks.register(self.plugin)

    # ------------------------------------------------------------------ buffers
    def _alloc_buffers(self, T: int) -> None:
        e = self.ecfg
        B = e.max_batch
        R = B + e.max_prefill_tokens // 1  # rows of the block table: decode + prefill requests
        R = min(R, 2 * B)
        S_max = 8
        self.rows_max = R
        self.layout = {}
        off = 0

        def reserve(name, n):
            nonlocal off
            self.layout[name] = (off, n)
            off += (n + 3) // 4 * 4  # keep 16-byte alignment of every field

        reserve("ids", T)
        reserve("pos", T)
        reserve("slot", T)
        reserve("block_table", R * self.max_pages_per_req)
        reserve("kv_lens", R)
        reserve("items", B * S_max * 4)
        reserve("merge_req", B)
        reserve("merge_begin", B + 1)
        reserve("tiles", (e.max_prefill_tokens // Q_TILE + B) * 4)
        reserve("sample_idx", 2 * B)
        self.packed_len = off
        # two pinned staging buffers (inputs) and two read-back buffers
        # (sampled tokens) alternate between consecutive steps, so the host can
        # plan step k + 1 while step k's copies are still queued
        self._hosts = [torch.zeros(off, dtype=torch.int32, pin_memory=True) for _ in range(2)]
        self._outs = [torch.zeros(2 * B, dtype=torch.int32, pin_memory=True) for _ in range(2)]
        self._h2d_done = [None, None]  # event after the copy that last read each staging buffer
        self._buf = 0
        self.host, self.out_host = self._hosts[0], self._outs[0]
        self.dev = torch.zeros(off, dtype=torch.int32, device=self.device)
        self.host_np = self.host.numpy()
        self.out_ids = torch.zeros(2 * B, dtype=torch.int32, device=self.device)
        self._timer_snap = None  # pinned copies of the timer rows of probe steps (created on first use)
        self.part_o = torch.zeros(B * S_max, self.cfg.n_q_heads // (self.tp.world if self.tp else 1),
                                  self.cfg.head_dim, dtype=torch.float32, device=self.device)
        self.part_lse = torch.zeros(B * S_max, self.part_o.shape[1], dtype=torch.float32, device=self.device)
        self.sample_idx64 = torch.zeros(2 * B, dtype=torch.int64, device=self.device)
        self.merge_cnt = torch.zeros(B * self.cfg.n_kv_heads, dtype=torch.int32, device=self.device)

    def new_scheduler(self, tier=None) -> Scheduler:
        """A scheduler with this engine's configuration (the engine's own, or
        a fresh one that simulates the engine's decisions without a model)."""
        e = self.ecfg
        capped = e.max_step_tokens > 0
        bucket = _weak_call(self, "_bucket")
        return Scheduler(e.num_pages, 16, e.max_batch, e.max_prefill_tokens, e.max_context, tier=tier,
                         max_step_tokens=e.max_step_tokens,
                         round_decode=(lambda nd: bucket(nd) or nd) if capped else None,
                         max_prefill_segments=MIXED_SEGMENTS if capped else 0,
                         prefix_cache=e.prefix_cache and tier is None and self.tier is None,
                         admission=e.admission if (e.admission != "lpm" or e.prefix_cache) else "fcfs")

    def _view(self, name, shape=None):
        o, n = self.layout[name]
        v = self.dev[o:o + n]
        return v.view(*shape) if shape is not None else v

    def _host(self, name):
        o, n = self.layout[name]
        return self.host_np[o:o + n]

    def _resident_prefix(self) -> int:
        try:
            return self.plane.r_for_kernel(self.cfg.group)
        except Exception:
            return self.sms

    def splits_for(self, n_decode: int) -> int:
        """KV splits per request: only when the (request, KV head) tasks leave
        SMs idle. A split task pays its own set-up and the merge of its
        partials, so on B200 one task per (request, head) beats splitting as
        soon as the tasks roughly fill the GPU (measured: 16 requests x 8
        heads x 1536 tokens take 40 us unsplit, 55 us in 3 splits)."""
        tasks = max(1, n_decode * self.hkv)
        return int(min(8, max(1, self.target_tasks // tasks)))

    # ------------------------------------------------------------------ public API
    def add_request(self, req: Request) -> None:
        self.sched.add(req)

    def abort(self, req: Request) -> bool:
        """Cancel a request between steps (pages freed, controller state
        dropped). Every tensor-parallel rank must abort the same requests
        before the same step."""
        ok = self.sched.abort(req)
        if ok:
            self.controller.forget([req.rid])
        return ok

    def add_prefilled(self, req: Request, first_token: int) -> None:
        """Admit ``req`` as if its prompt had been prefilled: its pages are
        allocated and left with whatever the cache holds there (see
        ``fill_kv_random``), and decoding starts from ``first_token``."""
        self.sched.admit_cached(req, first_token, self.clock)

    def fill_kv_random(self, seed: int = 0) -> None:
        """Fill every KV page with N(0, 1) values (synthetic contexts)."""
        g = torch.Generator(device=self.device)
        g.manual_seed(seed)
        for t in list(self.kv.k) + list(self.kv.v):
            t.normal_(generator=g)

    def has_work(self) -> bool:
        return not self.sched.idle

    # ------------------------------------------------------------------ planning
    def _mixed_pad(self, b: int) -> int:
        """Prefill rows of a fixed-shape mixed step with decode bucket ``b``:
        the scheduler's largest prefill budget for that bucket."""
        e = self.ecfg
        return min(e.max_prefill_tokens, max(e.max_step_tokens - b, 16))

    def _mixed_bucket(self, plan: StepPlan):
        """Decode bucket of a mixed step that fits the fixed shape, else None."""
        e = self.ecfg
        if e.max_step_tokens <= 0 or not e.mixed_graphs or self.tier is not None:
            return None
        nd = len(plan.decode)
        b = self._bucket(nd) if nd else 0
        if b is None or len(plan.prefill) > MIXED_SEGMENTS:
            return None
        if sum(n for _, _, n in plan.prefill) > self._mixed_pad(b):
            return None
        return b

    def _fill(self, plan: StepPlan, bucket: int | None, pad: int | None = None):
        """Write the step's inputs into the pinned staging buffer. ``pad``:
        a fixed-shape mixed step (prefill rows padded to ``pad`` tokens,
        prefill tiles and sampled rows to their bounds)."""
        e = self.ecfg
        dec = plan.decode
        nd = len(dec)
        ndp = bucket if bucket is not None else nd   # padded decode rows (graph bucket)
        pre = plan.prefill
        n_pre_tok = sum(n for _, _, n in pre)
        T = ndp + n_pre_tok
        ids, pos, slot = self._host("ids"), self._host("pos"), self._host("slot")
        mp = self.max_pages_per_req
        bt = self._host("block_table").reshape(-1, mp)
        kvl = self._host("kv_lens")
        # decode rows
        if self.tier is not None:
            self.tier.stage(dec)  # host-resident pages this step reads -> staging pages
        for i, r in enumerate(dec):
            p = r.total_len - 1
            tok = r.next_input_token()
            # a token the previous step sampled and the host has not read:
            # the embedding takes it from that step's output row on the device
            ids[i] = tok if tok != PENDING else -(1 + r._pending_row)
            pos[i] = p
            slot[i] = r.pages[p // 16] * 16 + p % 16  # the last page is always on the device
            pages = self.tier.pages_for(r) if self.tier is not None else r.pages
            npg = len(pages)
            bt[i, :npg] = pages
            kvl[i] = r.total_len
        if ndp > nd:  # padding rows: no cache write, empty attention items
            ids[nd:ndp] = 0
            pos[nd:ndp] = 0
            slot[nd:ndp] = -1
            kvl[nd:ndp] = 0
        # prefill rows
        row = ndp
        tiles = []
        for j, (r, start, n) in enumerate(pre):
            br = ndp + j
            ids[row:row + n] = r.prompt[start:start + n]
            pp = np.arange(start, start + n, dtype=np.int32)
            pos[row:row + n] = pp
            pg = np.asarray(r.pages, dtype=np.int32)
            slot[row:row + n] = pg[pp // 16] * 16 + pp % 16
            bt[br, :pg.size] = pg
            kvl[br] = start + n
            for t0 in range(0, n, Q_TILE):
                tiles.append((br, row - ndp + t0, min(Q_TILE, n - t0), start + t0))
            row += n
        tiles = order_prefill_tiles(tiles, e.prefill_order)
        if pad is not None:
            # padding rows: no cache write, in no attention tile, never sampled
            ids[row:ndp + pad] = 0
            pos[row:ndp + pad] = 0
            slot[row:ndp + pad] = -1
            T = ndp + pad
            n_tiles_max = -(-pad // Q_TILE) + MIXED_SEGMENTS - 1
            tiles += [(ndp, 0, 0, 0)] * (n_tiles_max - len(tiles))  # empty tiles (nq = 0)
        # decode plan
        S = self.splits_for(ndp) if ndp else 1
        n_items = 0
        if ndp:
            items, mreq, mbeg = native.plan_decode(kvl[:ndp].copy(), S)
            n_items = items.shape[0]
            self._host("items")[:n_items * 4] = items.reshape(-1)
            if S > 1:
                self._host("merge_req")[:ndp] = mreq
                self._host("merge_begin")[:ndp + 1] = mbeg
        th = self._host("tiles")
        for k, t in enumerate(tiles):
            th[4 * k:4 * k + 4] = t
        # sampled rows: every decode row (padded too), plus the last row of each finished prompt
        sidx = self._host("sample_idx")
        ns = ndp
        sidx[:ndp] = np.arange(ndp, dtype=np.int32)
        sample_map = [(r.rid, i) for i, r in enumerate(dec)]
        row = ndp
        for r, start, n in pre:
            if start + n >= r.prompt_len:
                sidx[ns] = row + n - 1
                sample_map.append((r.rid, ns))
                ns += 1
            row += n
        if pad is not None:
            sidx[ns:ndp + MIXED_SEGMENTS] = 0  # dummy rows, results ignored
            ns = ndp + MIXED_SEGMENTS
        return dict(T=T, nd=ndp, n_items=n_items, S=S, n_tiles=len(tiles), n_sample=ns,
                    sample_map=sample_map, n_real_decode=nd, pad=pad,
                    # for hooks that run after the next step was planned into the other buffer
                    items=self._host("items")[:n_items * 4].reshape(-1, 4).copy(),
                    kv_lens=kvl[:nd].tolist())

    def _batch(self, info, slots) -> ForwardBatch:
        mp = self.max_pages_per_req
        nd, S = info["nd"], info["S"]
        n_items = info["n_items"]
        return ForwardBatch(
            ids=self._view("ids"), pos=self._view("pos"), slot=self._view("slot"),
            n_tokens=info["T"], n_decode=nd,
            block_table=self._view("block_table", (-1, mp)), kv_lens=self._view("kv_lens"),
            items=self._view("items", (-1, 4)), n_items=n_items,
            part_o=self.part_o if S > 1 else None, part_lse=self.part_lse if S > 1 else None,
            merge_req=self._view("merge_req"), merge_begin=self._view("merge_begin"),
            n_merge=nd if S > 1 else 0, merge_cnt=self.merge_cnt if S > 1 else None, splits=S,
            tiles=self._view("tiles", (-1, 4)), n_tiles=info["n_tiles"],
            sample_idx=self.sample_idx64, n_sample=info["n_sample"], out_ids=self.out_ids,
            slots=slots, acquire=self._acq_code(), grid=self._grid(n_items * self.hkv),
            tier=self.tier if (self.tier is not None and nd > 0) else None,
        )

    def _grid(self, n_tasks: int) -> int:
        """CTAs of the decode launch: persistent (R) for static stride and
        ticket acquisition, one per task for cluster launch control (idle CTAs
        steal the unlaunched ones)."""
        if self.ecfg.acquire in ("static", "ticket") or not self.ecfg.levers:
            return max(1, min(self.R, n_tasks))
        return n_tasks

    def _acq_code(self) -> int:
        return {"static": 0, "ticket": 1, "clc": 2, "auto": 2}.get(self.ecfg.acquire, 0)

    # ------------------------------------------------------------------ levers
    def register_hook(self, hook) -> None:
        """Add a per-step hook (``on_batch_begin(engine, plan, info)`` /
        ``on_batch_end(engine, plan, info, ms)``); see engine/plugin.py."""
        self.hooks.register(hook)

    # ------------------------------------------------------------------ graphs
    def _bucket(self, nd: int) -> int | None:
        for b in DECODE_BUCKETS:
            if b >= nd and b <= self.ecfg.max_batch:
                return b
        return None

    def _graph_for(self, bucket, info, slots):
        g = self.graphs.get(bucket)
        if g is not None:
            return g
        batch = self._batch(info, slots)
        # a forward reads the previous step's sampled ids (decode inputs the
        # host has not seen) and overwrites them with its own: every warm-up
        # run starts from the same ids, and the replay too
        prev = self.out_ids.clone()
        s = torch.cuda.Stream(self.device)
        s.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(s):
            for _ in range(2):  # warm-up outside capture (lazy inits, attributes)
                self.out_ids.copy_(prev)
                self.model.forward(batch)
        torch.cuda.current_stream(self.device).wait_stream(s)
        graph = torch.cuda.CUDAGraph()
        if self._pool is None:
            self._pool = torch.cuda.graph_pool_handle()
        n0 = _ext.launches()
        with torch.cuda.graph(graph, pool=self._pool):
            self.model.forward(batch)
        self.out_ids.copy_(prev)
        self.graphs[bucket] = (graph, info["S"], info["n_items"], _ext.launches() - n0)
        return self.graphs[bucket]

    def warm_decode_graphs(self, sizes) -> list:
        """Capture the decode-step CUDA graphs for the buckets that hold the
        given decode batch sizes, before a timed or latency-sensitive run (a
        capture costs far more than a step). The capture runs on padding rows
        only: no cache writes, empty attention items. Every tensor-parallel
        rank must pass the same sizes (the graphs hold collectives)."""
        if not self.ecfg.cuda_graphs:
            return []
        self.drain()
        done = []
        for b in sorted({self._bucket(int(n)) for n in sizes if int(n) > 0} - {None}):
            if b in self.graphs:
                continue
            info = self._fill(StepPlan(), b)
            self.dev[: self.packed_len].copy_(self.host[: self.packed_len], non_blocking=True)
            self.sample_idx64[: info["n_sample"]].copy_(self._view("sample_idx")[: info["n_sample"]])
            self._graph_for(b, info, self.plane.slots() if self.ecfg.levers else None)
            done.append(b)
        torch.cuda.synchronize(self.device)
        return done

    # ------------------------------------------------------------------ step
    def _async_ok(self) -> bool:
        """Whether the host may run a step ahead of the device. Not with the
        tiered KV store (its page staging follows the host's plan) nor when
        every step must agree on the slowest rank's time (``clock_sync``)."""
        tp_sync = self.tp is not None and self.tp.world > 1 and self.ecfg.clock_sync
        return self.tier is None and not tp_sync

    def _use_buffers(self, k: int) -> None:
        self._buf = k
        self.host, self.out_host = self._hosts[k], self._outs[k]
        self.host_np = self.host.numpy()
        ev = self._h2d_done[k]
        if ev is not None:
            ev.synchronize()  # the copy that last read this staging buffer has run

    def _dispatch(self):
        """Plan and enqueue one step; its sampled tokens stay pending (-1 in
        the requests' outputs) until ``_resolve``. None when there is no work."""
        plan = self.sched.schedule()
        if plan.empty:
            return None
        nd = len(plan.decode)
        decode_only = not plan.prefill
        bucket = self._bucket(nd) if (decode_only and self.ecfg.cuda_graphs) else None
        mixed = None if decode_only else self._mixed_bucket(plan)
        self._use_buffers(self._buf ^ 1)
        if mixed is not None:
            info = self._fill(plan, mixed, pad=self._mixed_pad(mixed))
            key = ("mixed", mixed) if self.ecfg.cuda_graphs else None
        else:
            info = self._fill(plan, bucket)
            key = bucket
        if key is not None and self.tier is not None and self.tier.stage_mode == "copy" and self.tier.last_stage:
            # copy-mode staging issues one cudaMemcpyAsync per run of host
            # pages, planned on the host for this step: a graph would replay
            # the runs of the step it was captured in, so such steps run eagerly
            # (the zero-copy kernel reads its page pairs from device memory and
            # replays correctly)
            key = None
        slots = self.plane.slots() if self.ecfg.levers else None
        self.hooks.begin(self, plan, info)
        stream = torch.cuda.current_stream(self.device)
        # one H2D copy of every step input
        self.dev[: self.packed_len].copy_(self.host[: self.packed_len], non_blocking=True)
        h2d = torch.cuda.Event()
        h2d.record(stream)
        self._h2d_done[self._buf] = h2d
        si = self._view("sample_idx")
        self.sample_idx64[: info["n_sample"]].copy_(si[: info["n_sample"]])
        ev0 = torch.cuda.Event(enable_timing=True)
        ev1 = torch.cuda.Event(enable_timing=True)
        ev0.record(stream)
        used_graph = False
        if key is not None:
            graph, S, n_items, n_launch = self._graph_for(key, info, slots)
            assert S == info["S"] and n_items == info["n_items"]
            graph.replay()
            self.graph_launches += n_launch
            used_graph = True
        else:
            self.model.forward(self._batch(info, slots))
        ev1.record(stream)
        if info.get("probe"):
            # the timer rows of this step, before a later step clears them
            n = info["n_items"] * self.hkv
            if self._timer_snap is None:
                self._timer_snap = [torch.zeros(self.plane.N, dtype=torch.int64, pin_memory=True) for _ in range(2)]
            snap = self._timer_snap[self._buf][:n]
            snap.copy_(self.plane.timer_t[:n], non_blocking=True)
            info["timer"] = snap
        ns = info["n_sample"]
        self.out_host[:ns].copy_(self.out_ids[:ns], non_blocking=True)
        done_ev = torch.cuda.Event()
        done_ev.record(stream)
        # the step's tokens are pending: counts advance now (so the next step
        # can be planned), values arrive in _resolve
        by_rid = {r.rid: r for r in plan.decode}
        by_rid.update({r.rid: r for r, _, _ in plan.prefill})
        rows = [(by_rid[rid], row) for rid, row in info["sample_map"]]
        finished = self.sched.commit(plan, {req.rid: PENDING for req, _ in rows}, float("nan"))
        pend = []
        for req, row in rows:
            pend.append((req, len(req.output) - 1, row))
            req._pending_row = row
        self._inflight.append(_InFlight(plan, info, ev0, ev1, done_ev, self._buf, pend, used_graph, finished))
        self.step_no += 1
        return plan

    def _resolve(self, f: "_InFlight") -> list:
        """Wait for an enqueued step, write its tokens into the requests and
        finish its bookkeeping. Returns the requests it finished."""
        f.done_ev.synchronize()
        ms = f.ev0.elapsed_time(f.ev1)
        if self.tp is not None and self.tp.world > 1 and self.ecfg.clock_sync:
            # every tensor-parallel rank must make the same scheduling
            # decisions (admissions follow the workload clock): advance all
            # clocks by the slowest rank's step time
            ms = self.tp.max_over_ranks(ms)
        self.clock += ms / 1e3
        out = self._outs[f.buf].numpy()
        for req, idx, row in f.pend:
            req.output[idx] = int(out[row])
            req.token_times[idx] = self.clock
            if idx == len(req.output) - 1:
                req._pending_row = None
        self.hooks.end(self, f.plan, f.info, ms)
        if f.finished:
            self.controller.forget([r.rid for r in f.finished])
        self.stats.append(StepStats(len(f.plan.decode), f.plan.n_tokens - len(f.plan.decode), ms, f.graph))
        return f.finished

    def drain(self) -> list:
        """Wait for every enqueued step and apply its tokens; returns the
        requests they finished."""
        done = []
        while self._inflight:
            done += self._resolve(self._inflight.popleft())
        return done

    def step(self) -> tuple[StepPlan, list]:
        """One step, synchronously: plan it, run it, read its sampled tokens
        back. Returns (plan, requests it finished)."""
        done = self.drain()
        plan = self._dispatch()
        done += self.drain()
        return (plan if plan is not None else StepPlan()), done

    def step_async(self) -> tuple[StepPlan, list]:
        """One step with the host a step ahead of the device: plan and
        enqueue step k (decode inputs that step k - 1 samples are read on the
        device), then wait for step k - 1 and apply its tokens, so the host's
        planning of k overlaps the device's work on k - 1. Returns (plan of
        step k, requests finished by the steps read back in this call);
        ``drain()`` reads back the step still in flight. Falls back to
        ``step()`` where the host may not run ahead (``_async_ok``)."""
        if not self._async_ok():
            return self.step()
        plan = self._dispatch()
        keep = 1 if plan is not None else 0
        done = []
        while len(self._inflight) > keep:
            done += self._resolve(self._inflight.popleft())
        return (plan if plan is not None else StepPlan()), done

    def _before_preempt(self) -> None:
        """A preempted request's generated tokens become part of its prompt,
        so their values must be on the host: read back every step in flight."""
        self.drain()

    # ------------------------------------------------------------------ convenience
    def generate(self, prompts, max_new_tokens: int = 16) -> list:
        """Greedy generation for a list of prompts (token id arrays)."""
        reqs = [Request(rid=i, prompt=np.asarray(p, dtype=np.int32), max_new_tokens=max_new_tokens)
                for i, p in enumerate(prompts)]
        for r in reqs:
            self.add_request(r)
        while self.has_work():
            self.step_async()
        self.drain()
        return [r.output for r in reqs]
