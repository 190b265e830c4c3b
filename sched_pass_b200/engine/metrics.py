"""Prometheus metrics of the serving engine (exposed by the HTTP server at
``GET /metrics``).

Per server instance (its own registry, so several engines in one process do
not collide):

* counters: engine steps, decode tokens, prefill tokens, finished requests;
* histograms: device time of each engine step (ms), per-request TPOT (ms),
  TTFT (s, on the engine's workload clock) and end-to-end latency (s, host
  clock of the HTTP side);
* gauges read at scrape time: queued and running requests, and the
  scheduling plugin's counters (plans, timer probes, CLC armings, hook
  errors).

The reference reports the same quantities as a periodic log line and a
load-generator summary (python/sched_sglang_plugin.py:308-314,
python/sched_trace_loadgen.py:130-142); a scrape endpoint carries them to a
monitoring system while the server runs.
"""
from __future__ import annotations

STEP_MS_BUCKETS = (0.5, 1, 2, 3, 4, 5, 6, 8, 10, 15, 20, 30, 50, 100, 200, 500)
TPOT_MS_BUCKETS = (1, 2, 3, 4, 5, 6, 8, 10, 15, 20, 30, 50, 100, 250, 1000)
SECONDS_BUCKETS = (0.01, 0.025, 0.05, 0.1, 0.25, 0.5, 1, 2.5, 5, 10, 30, 60)


class ServerMetrics:
    def __init__(self, server):
        from prometheus_client import CollectorRegistry, Counter, Gauge, Histogram

        self.registry = r = CollectorRegistry()
        self.steps = Counter("sched_engine_steps", "Engine steps run", registry=r)
        self.decode_tokens = Counter("sched_engine_decode_tokens", "Tokens produced by decode rows", registry=r)
        self.prefill_tokens = Counter("sched_engine_prefill_tokens", "Prompt tokens prefilled", registry=r)
        self.finished = Counter("sched_requests_finished", "Requests completed", registry=r)
        self.step_ms = Histogram("sched_engine_step_ms", "Device time of one engine step (ms)",
                                 buckets=STEP_MS_BUCKETS, registry=r)
        self.tpot_ms = Histogram("sched_request_tpot_ms", "Mean time per output token after the first (ms)",
                                 buckets=TPOT_MS_BUCKETS, registry=r)
        self.ttft_s = Histogram("sched_request_ttft_seconds", "Time to first token on the workload clock (s)",
                                buckets=SECONDS_BUCKETS, registry=r)
        self.e2e_s = Histogram("sched_request_e2e_seconds", "Submit-to-completion latency, host clock (s)",
                               buckets=SECONDS_BUCKETS, registry=r)
        Gauge("sched_requests_queued", "Requests waiting for admission", registry=r).set_function(
            lambda: server._inbox.qsize())
        Gauge("sched_requests_running", "Admitted requests not yet finished", registry=r).set_function(
            lambda: len(server._pending))
        eng = server.engine

        def plugin_value(name):
            def read():
                p = getattr(eng, "plugin", None)
                if p is None:
                    return 0.0
                if name == "hook_errors":
                    return float(getattr(getattr(eng, "hooks", None), "errors", 0))
                return float(getattr(p.stats, name, 0))
            return read

        def cache_value(name):
            def read():
                c = getattr(getattr(eng, "sched", None), "cache", None)
                return float(getattr(c, name, 0)) if c is not None else 0.0
            return read

        Gauge("sched_prefix_cache_hit_tokens", "Prompt tokens served from cached KV pages",
              registry=r).set_function(cache_value("hits"))
        Gauge("sched_prefix_cache_lookup_tokens", "Prompt tokens looked up in the prefix cache",
              registry=r).set_function(cache_value("lookups"))
        for name, doc in (("planned", "Steps whose task order was re-planned"),
                          ("probes", "Steps with the per-task timer armed"),
                          ("clc_armed", "Steps with cluster launch control armed"),
                          ("hook_errors", "Scheduling hook errors (isolated, never fatal)")):
            Gauge(f"sched_plugin_{name}", doc, registry=r).set_function(plugin_value(name))

    def on_step(self, engine, plan) -> None:
        self.steps.inc()
        self.decode_tokens.inc(len(plan.decode))
        self.prefill_tokens.inc(sum(n for _, _, n in plan.prefill))
        stats = getattr(engine, "stats", None)
        if stats:
            self.step_ms.observe(float(stats[-1].device_ms))

    def on_done(self, tpot_s, ttft_s, e2e_s) -> None:
        self.finished.inc()
        if tpot_s is not None:
            self.tpot_ms.observe(1e3 * tpot_s)
        if ttft_s is not None:
            self.ttft_s.observe(ttft_s)
        self.e2e_s.observe(e2e_s)

    def text(self) -> bytes:
        from prometheus_client import generate_latest
        return generate_latest(self.registry)
