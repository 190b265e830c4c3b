"""HTTP front end of the serving engine.

``EngineServer`` owns an engine and runs it on a dedicated thread (the only
thread that touches the GPU): HTTP handlers enqueue requests and wait for
their completion; the engine thread admits queued requests between steps,
steps while there is work, and completes finished requests. Endpoints:

* ``POST /generate`` -- ``{"input_ids": [...], "sampling_params":
  {"max_new_tokens": N}}`` (the ``/generate`` shape SGLang-style clients
  and ``engine/loadgen.py`` send); returns ``{"output_ids": [...],
  "meta_info": {"prompt_tokens", "completion_tokens", "e2e_latency",
  "ttft", "tpot"}}``. Decoding is greedy and runs ``max_new_tokens`` tokens.
  An optional ``"rid"`` (any string) names the request for ``/abort``;
  ``"stream": true`` answers with server-sent events instead, one
  ``data: {"index": i, "token": t}`` per generated token as the engine
  produces it and a final ``data: {"done": true, "meta_info": {...}}``.
* ``POST /abort`` -- ``{"rid": ...}``: cancel a queued or running request
  between steps (its pages are freed; its ``/generate`` call answers 499).
* ``GET /health`` -- liveness plus queue depths.
* ``GET /stats`` -- steps, decode tokens, the scheduling plugin's counters.
* ``GET /metrics`` -- the same and step-time / TPOT / TTFT / latency
  histograms in the Prometheus text format (``engine/metrics.py``).

    python -m sched_pass_b200.engine.server --model llama-3-8b --port 30000
    # tensor parallel: rank 0 serves HTTP, the other ranks follow
    python -m torch.distributed.run --nproc-per-node 8 --master-addr 127.0.0.1 \
        -m sched_pass_b200.engine.server --model llama-3-8b --port 30000
"""
from __future__ import annotations

import argparse
import collections
import concurrent.futures as cf
import json
import math
import queue
import threading
import time

import numpy as np


def latency_summary(lat: list) -> dict:
    """p50 / p99 of TPOT and TTFT (ms) over finished requests, given as
    (tpot s or None, ttft s or None) pairs (nearest-rank percentiles)."""
    def pct(v, q):
        v = sorted(v)
        return round(1e3 * v[min(len(v) - 1, max(0, math.ceil(q * len(v)) - 1))], 3) if v else None
    tpot = [a for a, _ in lat if a is not None]
    ttft = [b for _, b in lat if b is not None]
    return {"finished": len(lat), "tpot_ms_p50": pct(tpot, 0.5), "tpot_ms_p99": pct(tpot, 0.99),
            "ttft_ms_p50": pct(ttft, 0.5), "ttft_ms_p99": pct(ttft, 0.99)}


class EngineServer:
    def __init__(self, engine, idle_wait_s: float = 0.002):
        self.engine = engine
        self.idle_wait_s = idle_wait_s
        self._inbox: queue.Queue = queue.Queue()
        self._pending: dict = {}
        self._next_rid = 0
        self._aborts: queue.Queue = queue.Queue()
        self._dropped: set = set()
        self._named: dict = {}  # client rid -> internal rid
        self._lock = threading.Lock()
        self._stop = threading.Event()
        self._thread: threading.Thread | None = None
        self.steps = 0
        self.decode_tokens = 0
        self.error: BaseException | None = None
        # (tpot s or None, ttft s or None) of the most recently finished requests
        self._latencies: collections.deque = collections.deque(maxlen=4096)
        try:
            from .metrics import ServerMetrics
            self.metrics = ServerMetrics(self)
        except ImportError:  # prometheus_client absent: /metrics answers 404
            self.metrics = None

    # ---------------------------------------------------------------- client side
    def submit(self, input_ids, max_new_tokens: int, urgency: float = 0.0, name: str | None = None,
               stream: bool = False) -> cf.Future:
        """Queue one request; the future resolves to the response dict.
        ``name``: a client id that ``cancel`` accepts. ``stream``: the
        request's tokens are also put, as they are produced, on
        ``future.tokens`` (a queue.Queue; None marks the end)."""
        from .request import Request
        ids = np.asarray(input_ids, dtype=np.int32)
        if ids.ndim != 1 or ids.size == 0:
            raise ValueError("input_ids must be a non-empty list of token ids")
        if max_new_tokens < 1:
            raise ValueError("max_new_tokens must be >= 1")
        fut: cf.Future = cf.Future()
        req = Request(rid=-1, prompt=ids, max_new_tokens=int(max_new_tokens), urgency=float(urgency))
        req._t_submit = time.perf_counter()  # host clock of the HTTP side
        req._name = None if name is None else str(name)
        req._stream = queue.Queue() if stream else None
        req._sent = 0
        fut.tokens = req._stream
        with self._lock:
            # under the lock that _die takes: a request is either refused here
            # or queued before the engine thread drains the queue on its way out
            if self.error is not None:
                self._fail(req, fut, RuntimeError(f"the engine stopped on an error: {self.error!r}"))
                return fut
            req.rid = self._next_rid
            self._next_rid += 1
            if name is not None:
                self._named[str(name)] = req.rid
            self._inbox.put((req, fut))
        return fut

    def cancel(self, name) -> None:
        """Ask the engine thread to abort the request submitted as ``name``
        (a client id) or with internal id ``name`` (an int)."""
        with self._lock:
            rid = self._named.pop(str(name), None) if not isinstance(name, int) else name
        if rid is None:
            raise KeyError(f"no request named {name!r}")
        self._aborts.put(rid)

    # ---------------------------------------------------------------- engine thread
    @staticmethod
    def _end_stream(req) -> None:
        if getattr(req, "_stream", None) is not None:
            req._stream.put(None)

    def _fail(self, req, fut, exc) -> None:
        """Fail one request: its stream ends and its future raises."""
        self._end_stream(req)
        if not fut.done():
            fut.set_exception(exc)

    def _die(self, exc: BaseException) -> None:
        """The engine thread ends on an error: every request it holds, admitted
        or still queued, fails (its stream ends and its future raises), and
        later submissions fail at once (``submit`` checks ``error``)."""
        with self._lock:
            self.error = exc
            queued = []
            while True:
                try:
                    queued.append(self._inbox.get_nowait())
                except queue.Empty:
                    break
        for req, fut in list(self._pending.values()) + queued:
            self._fail(req, fut, exc)
        self._pending.clear()

    def _drain_aborts(self) -> list:
        rids = []
        while True:
            try:
                rids.append(self._aborts.get_nowait())
            except queue.Empty:
                return rids

    def _apply_aborts(self, rids) -> None:
        """Abort on the engine (between steps) and fail the callers."""
        for rid in rids:
            item = self._pending.pop(rid, None)
            if item is None:
                # still in the inbox: it will be dropped when admitted
                self._dropped.add(rid)
                continue
            req, fut = item
            self.engine.abort(req)
            self._fail(req, fut, cf.CancelledError(f"request {rid} aborted"))

    def _admit(self) -> None:
        while True:
            try:
                req, fut = self._inbox.get_nowait()
            except queue.Empty:
                return
            if req.rid in self._dropped:
                self._dropped.discard(req.rid)
                self._fail(req, fut, cf.CancelledError(f"request {req.rid} aborted"))
                continue
            req.arrival = self.engine.clock
            try:
                self.engine.add_request(req)
            except Exception as e:  # noqa: BLE001 - a bad request fails alone
                self._fail(req, fut, e)
                continue
            self._pending[req.rid] = (req, fut)

    def _push_tokens(self, plan) -> None:
        """Stream the tokens a step produced (requests submitted with stream)."""
        for r in list(plan.decode) + [r for r, _, _ in plan.prefill]:
            q = getattr(r, "_stream", None)
            if q is None:
                continue
            if len(r.output) < r._sent:  # preempted: its streamed tokens moved into the prompt
                r._sent = 0
            base = getattr(r, "_streamed_total", 0)
            for t in r.output[r._sent:]:
                q.put((base, int(t)))
                base += 1
            r._streamed_total = base
            r._sent = len(r.output)

    def _complete(self, done) -> None:
        now = time.perf_counter()
        for r in done:
            if getattr(r, "_stream", None) is not None:
                r._stream.put(None)
            item = self._pending.pop(r.rid, None)
            if item is None:
                continue
            _, fut = item
            if getattr(r, "_name", None) is not None:
                with self._lock:
                    self._named.pop(r._name, None)
            tpot = r.tpot()
            self._latencies.append((tpot, r.ttft()))
            if self.metrics is not None:
                self.metrics.on_done(tpot, r.ttft(), now - r._t_submit)
            fut.set_result({
                "output_ids": [int(t) for t in r.output],
                "meta_info": {"prompt_tokens": r.prompt_len, "completion_tokens": len(r.output),
                              "e2e_latency": now - r._t_submit, "ttft": r.ttft(), "tpot": tpot,
                              "preemptions": r.preemptions},
            })

    def _loop(self) -> None:
        try:
            dev = getattr(self.engine, "device", None)
            if dev is not None and getattr(dev, "type", "") == "cuda":
                import torch
                torch.cuda.set_device(dev)
            while not self._stop.is_set():
                self._apply_aborts(self._drain_aborts())
                self._admit()
                if self.engine.has_work():
                    plan, done = self.engine.step()
                    self.steps += 1
                    self.decode_tokens += len(plan.decode)
                    if self.metrics is not None:
                        self.metrics.on_step(self.engine, plan)
                    self._push_tokens(plan)
                    self._complete(done)
                else:
                    try:
                        item = self._inbox.get(timeout=self.idle_wait_s)
                        self._inbox.put(item)
                    except queue.Empty:
                        pass
        except BaseException as e:  # noqa: BLE001 - report to every waiter
            self._die(e)

    def start(self) -> "EngineServer":
        if self._thread is None:
            self._thread = threading.Thread(target=self._loop, name="sched-engine", daemon=True)
            self._thread.start()
        return self

    def stop(self, timeout: float = 10.0) -> None:
        self._stop.set()
        if self._thread is not None:
            self._thread.join(timeout)
            self._thread = None

    # ---------------------------------------------------------------- HTTP
    def app(self):
        import asyncio

        from fastapi import FastAPI, HTTPException
        from fastapi.responses import JSONResponse, Response, StreamingResponse

        app = FastAPI(title="sched_pass_b200")

        @app.post("/generate")
        async def generate(body: dict):
            ids = body.get("input_ids")
            sp = body.get("sampling_params") or {}
            if ids is None:
                raise HTTPException(400, "input_ids is required (token ids; no tokenizer in this server)")
            stream = bool(body.get("stream", False))
            try:
                fut = self.submit(ids, int(sp.get("max_new_tokens", 16)), float(body.get("urgency", 0.0)),
                                  name=body.get("rid"), stream=stream)
            except ValueError as e:
                raise HTTPException(400, str(e)) from e
            if stream:
                async def events():
                    while True:
                        item = await asyncio.to_thread(fut.tokens.get)
                        if item is None:
                            break
                        yield f"data: {json.dumps({'index': item[0], 'token': item[1]})}\n\n"
                    try:
                        res = await asyncio.wrap_future(fut)
                        yield f"data: {json.dumps({'done': True, 'meta_info': res['meta_info']})}\n\n"
                    except Exception as e:  # noqa: BLE001 - aborted or failed mid-stream
                        yield f"data: {json.dumps({'done': True, 'error': repr(e)})}\n\n"
                return StreamingResponse(events(), media_type="text/event-stream")
            try:
                return JSONResponse(await asyncio.wrap_future(fut))
            except (cf.CancelledError, asyncio.CancelledError) as e:
                raise HTTPException(499, f"aborted: {e}") from e
            except Exception as e:  # noqa: BLE001
                raise HTTPException(500, repr(e)) from e

        @app.post("/abort")
        async def abort(body: dict):
            try:
                self.cancel(body.get("rid"))
            except KeyError as e:
                raise HTTPException(404, str(e)) from e
            return {"ok": True}

        @app.get("/health")
        async def health():
            return {"ok": self.error is None, "queued": self._inbox.qsize(), "running": len(self._pending)}

        @app.get("/stats")
        async def stats():
            out = {"steps": self.steps, "decode_tokens": self.decode_tokens, "queued": self._inbox.qsize(),
                   "running": len(self._pending)}
            stats = getattr(self.engine, "stats", None)
            if stats:
                from .engine import summarize_steps
                out["engine"] = summarize_steps(list(stats[-4096:]))
            out["requests"] = latency_summary(list(self._latencies))
            cache = getattr(getattr(self.engine, "sched", None), "cache", None)
            if cache is not None:
                out["prefix_cache"] = {"hit_tokens": cache.hits, "lookup_tokens": cache.lookups,
                                       "cached_pages": len(cache.key_of), "evictable_pages": cache.evictable}
            plugin = getattr(self.engine, "plugin", None)
            if plugin is not None:
                s = plugin.stats
                out["sched"] = {"planned": s.planned, "probes": s.probes, "clc_armed": s.clc_armed,
                                "orders": s.orders, "hook_errors": self.engine.hooks.errors}
            return out

        @app.get("/metrics")
        async def metrics():
            if self.metrics is None:
                raise HTTPException(404, "prometheus_client is not installed")
            return Response(self.metrics.text(), media_type="text/plain; version=0.0.4; charset=utf-8")

        return app

    def serve(self, host: str = "127.0.0.1", port: int = 30000, log_level: str = "warning") -> None:
        import uvicorn
        self.start()
        try:
            uvicorn.run(self.app(), host=host, port=port, log_level=log_level)
        finally:
            self.stop()


class TPEngineServer(EngineServer):
    """HTTP front end of a tensor-parallel engine: rank 0 of the group runs
    this server, every other rank runs ``follow`` with its own engine shard.

    Each iteration rank 0 admits the requests submitted since the last one
    (requests its engine refuses fail alone and are not sent), broadcasts
    them with a stop flag to the group, and every rank adds the same
    requests and then steps: the ranks' schedulers see identical admissions,
    so every rank issues the same collectives in the same order (the engine
    already advances every rank's workload clock by the slowest rank's step
    time). Only the engine thread of rank 0 talks to the group."""

    def __init__(self, engine, group=None, idle_wait_s: float = 0.002, heartbeat=None):
        super().__init__(engine, idle_wait_s)
        self.group = group
        # parallel.health.Heartbeat: a silent or departed rank ends the loop
        # (RankFailure, pending requests failed) before the next broadcast
        self.heartbeat = heartbeat

    def _admit_batch(self) -> list:
        sent = []
        while True:
            try:
                req, fut = self._inbox.get_nowait()
            except queue.Empty:
                break
            if req.rid in self._dropped:
                self._dropped.discard(req.rid)
                self._fail(req, fut, cf.CancelledError(f"request {req.rid} aborted"))
                continue
            req.arrival = self.engine.clock
            try:
                self.engine.add_request(req)
            except Exception as e:  # noqa: BLE001 - a bad request fails alone, on rank 0 only
                self._fail(req, fut, e)
                continue
            self._pending[req.rid] = (req, fut)
            sent.append((req.rid, [int(t) for t in req.prompt], req.max_new_tokens, req.urgency))
        return sent

    def _loop(self) -> None:
        import torch.distributed as dist
        try:
            dev = getattr(self.engine, "device", None)
            if dev is not None and getattr(dev, "type", "") == "cuda":
                import torch
                torch.cuda.set_device(dev)
            while True:
                if not self.engine.has_work() and self._inbox.empty() and not self._stop.is_set():
                    try:  # idle: wait briefly for a request before the next round
                        item = self._inbox.get(timeout=self.idle_wait_s)
                        self._inbox.put(item)
                    except queue.Empty:
                        pass
                if self.heartbeat is not None:
                    self.heartbeat.check()
                stop = self._stop.is_set()
                aborts = [] if stop else [r for r in self._drain_aborts()]
                # only requests every rank holds are aborted on the group
                held = [r for r in aborts if r in self._pending]
                self._apply_aborts(aborts)
                msg = [{"stop": stop, "reqs": [] if stop else self._admit_batch(), "aborts": held}]
                dist.broadcast_object_list(msg, src=dist.get_global_rank(self.group, 0) if self.group else 0,
                                           group=self.group)
                if stop:
                    break
                if self.engine.has_work():
                    plan, done = self.engine.step()
                    self.steps += 1
                    self.decode_tokens += len(plan.decode)
                    if self.metrics is not None:
                        self.metrics.on_step(self.engine, plan)
                    self._push_tokens(plan)
                    self._complete(done)
        except BaseException as e:  # noqa: BLE001 - report to every waiter
            self._die(e)


def follow(engine, group=None, heartbeat=None, max_rounds: int | None = None) -> int:
    """The loop of a non-zero rank of a tensor-parallel server: receive each
    round's admitted requests from rank 0, add them, step. Returns the number
    of steps taken when rank 0 broadcasts stop (or after ``max_rounds``
    rounds). With a ``heartbeat`` a silent peer raises RankFailure before the
    next round; a peer lost during a round ends it with the process group's
    timeout."""
    import torch.distributed as dist

    from .request import Request
    dev = getattr(engine, "device", None)
    if dev is not None and getattr(dev, "type", "") == "cuda":
        import torch
        torch.cuda.set_device(dev)
    src = dist.get_global_rank(group, 0) if group else 0
    steps = 0
    rounds = 0
    held = {}  # rid -> Request this rank admitted (finished ones are dropped as they finish)
    while max_rounds is None or rounds < max_rounds:
        rounds += 1
        if heartbeat is not None:
            heartbeat.check()
        msg = [None]
        dist.broadcast_object_list(msg, src=src, group=group)
        for rid in msg[0].get("aborts", []):
            req = held.pop(rid, None)
            if req is not None:
                engine.abort(req)
        for rid, ids, max_new, urgency in msg[0]["reqs"]:
            req = Request(rid=rid, prompt=np.asarray(ids, dtype=np.int32), max_new_tokens=max_new,
                          urgency=urgency, arrival=engine.clock)
            held[rid] = req
            engine.add_request(req)
        if msg[0]["stop"]:
            return steps
        if engine.has_work():
            _, done = engine.step()
            for r in done:
                held.pop(r.rid, None)
            steps += 1
    return steps


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="llama-3-8b")
    ap.add_argument("--host", default="127.0.0.1")
    ap.add_argument("--port", type=int, default=30000)
    ap.add_argument("--max-batch", type=int, default=128)
    ap.add_argument("--max-context", type=int, default=4096)
    ap.add_argument("--acquire", default="auto")
    ap.add_argument("--tp-mode", default=None, choices=[None, "fused", "sp", "nccl"])
    ap.add_argument("--prefix-cache", action="store_true", help="share KV pages of common prompt prefixes")
    ap.add_argument("--admission", default="fcfs", choices=["fcfs", "urgency", "lpm"])
    ap.add_argument("--config", help="YAML/JSON file with engine: and sched: sections (replaces the flags above)")
    a = ap.parse_args(argv)
    import torch

    from ..models.config import get_config
    from ..parallel.tp import TensorParallel, init_distributed
    from .engine import Engine, EngineConfig
    rank, world, local = init_distributed("nccl")  # torchrun's env; world 1 without it
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    tp = TensorParallel(mode=a.tp_mode, device=dev) if world > 1 else None
    if a.config:
        from .config_file import apply_sched_env, load_config
        ecfg, scfg = load_config(a.config)
        apply_sched_env(scfg)  # the plugin reads its knobs from SCHED_*
        ecfg.verbose = ecfg.verbose and rank == 0
    else:
        ecfg = EngineConfig(max_batch=a.max_batch, max_context=a.max_context, acquire=a.acquire,
                            verbose=rank == 0, prefix_cache=a.prefix_cache, admission=a.admission)
    eng = Engine(get_config(a.model), ecfg, dev, tp=tp)
    if world == 1:
        EngineServer(eng).serve(a.host, a.port)
        return 0
    from ..parallel.health import Heartbeat
    hb = Heartbeat(rank, world).start()
    if rank == 0:
        TPEngineServer(eng, heartbeat=hb).serve(a.host, a.port)
    else:
        follow(eng, heartbeat=hb)
    hb.stop()
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
