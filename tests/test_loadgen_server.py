"""Load generator and HTTP server on the CPU, with a fake model behind the
real scheduler (continuous batching, chunked prefill, page accounting)."""
import json
import socket
import threading
import time

import numpy as np

from sched_pass_b200.engine import loadgen
from sched_pass_b200.engine.scheduler import Scheduler
from sched_pass_b200.engine.server import EngineServer


class FakeEngine:
    """Engine interface over the real Scheduler; the 'model' emits
    (previous token + 1) mod vocab and every step takes 1 ms of clock."""

    def __init__(self, vocab=1000, num_pages=4096, max_batch=16, max_prefill=256, max_context=4096):
        self.sched = Scheduler(num_pages, 16, max_batch, max_prefill, max_context)
        self.clock = 0.0
        self.vocab = vocab
        self.device = None
        self.step_no = 0

    def add_request(self, r):
        self.sched.add(r)

    def abort(self, r):
        return self.sched.abort(r)

    def has_work(self):
        return not self.sched.idle

    def step(self):
        plan = self.sched.schedule()
        sampled = {}
        for r in plan.decode:
            sampled[r.rid] = (r.next_input_token() + 1) % self.vocab
        for r, start, n in plan.prefill:
            if start + n >= r.prompt_len:
                sampled[r.rid] = (int(r.prompt[-1]) + 1) % self.vocab
        self.clock += 0.001
        done = self.sched.commit(plan, sampled, self.clock)
        self.step_no += 1
        return plan, done


def test_inprocess_run_completes_everything():
    work = loadgen.dispersed(40, mu=4.0, sigma=0.8, lo=8, hi=300, out=5, vocab=1000, seed=1, rate=200.0)
    eng = FakeEngine()
    res, wall = loadgen.run_inprocess(eng, work)
    assert all(r.ok for r in res) and all(r.n_out == 5 for r in res)
    s = loadgen.summarize(res, wall)
    assert s["n_ok"] == 40 and s["tpot_p50"] is not None and s["tpot_p50"] >= 0.001 - 1e-9


def test_trace_roundtrip_with_truncated_tail(tmp_path):
    p = tmp_path / "t.jsonl"
    recs = [{"chat_id": i, "timestamp": 0.5 * i, "input_length": 20 + 7 * i, "output_length": 3,
             "hash_ids": [100 + j for j in range(i + 2)]} for i in range(6)]
    text = "\n".join(json.dumps(r) for r in recs) + "\n" + '{"chat_id": 99, "timest'
    p.write_text(text)
    got = loadgen.load_trace(str(p))
    assert len(got) == 6
    work = loadgen.from_trace(got, vocab=1000, speed=2.0)
    assert [len(w.prompt) for w in work] == [20 + 7 * i for i in range(6)]
    assert work[3].arrival == 0.75
    # shared hash prefix -> shared token prefix
    assert np.array_equal(work[2].prompt[:32], work[4].prompt[:32])
    assert loadgen.selftest(str(p)) == 0


def test_server_futures_and_http_replay():
    srv = EngineServer(FakeEngine()).start()
    try:
        futs = [srv.submit([1, 2, 3], 4), srv.submit(list(range(50)), 2)]
        outs = [f.result(timeout=10) for f in futs]
        assert outs[0]["output_ids"] == [4, 5, 6, 7]
        assert outs[1]["output_ids"] == [50, 51]
        assert outs[0]["meta_info"]["completion_tokens"] == 4
        try:
            srv.submit([], 3)
        except ValueError:
            pass
        else:
            raise AssertionError("empty prompt accepted")

        import uvicorn
        with socket.socket() as s:
            s.bind(("127.0.0.1", 0))
            port = s.getsockname()[1]
        server = uvicorn.Server(uvicorn.Config(srv.app(), host="127.0.0.1", port=port, log_level="error"))
        th = threading.Thread(target=server.run, daemon=True)
        th.start()
        for _ in range(200):
            if server.started:
                break
            time.sleep(0.02)
        assert server.started
        work = loadgen.dispersed(24, mu=3.5, sigma=0.5, lo=4, hi=64, out=3, vocab=1000, seed=2)
        res, wall = loadgen.replay_http(f"http://127.0.0.1:{port}", work, concurrency=8, realtime=False)
        assert all(r.ok and r.n_out == 3 for r in res)
        sres, _ = loadgen.replay_http(f"http://127.0.0.1:{port}", work[:6], concurrency=4, realtime=False,
                                      stream=True)
        assert all(r.ok and r.n_out == 3 and r.ttft is not None and r.tpot is not None for r in sres)
        import requests
        st = requests.get(f"http://127.0.0.1:{port}/stats", timeout=5).json()
        assert st["steps"] > 0 and st["decode_tokens"] > 0
        rq = st["requests"]
        assert rq["finished"] == 32 and rq["tpot_ms_p50"] is not None and rq["ttft_ms_p99"] >= rq["ttft_ms_p50"]
        assert requests.get(f"http://127.0.0.1:{port}/health", timeout=5).json()["ok"]
        m = requests.get(f"http://127.0.0.1:{port}/metrics", timeout=5)
        assert m.status_code == 200
        vals = {}
        for line in m.text.splitlines():
            if line and not line.startswith("#"):
                k, v = line.rsplit(" ", 1)
                vals[k] = float(v)
        assert vals["sched_engine_steps_total"] == st["steps"] > 0
        assert vals["sched_requests_finished_total"] == 32  # 2 submitted directly + 24 + 6 replayed
        assert vals["sched_request_tpot_ms_count"] == 32 and vals["sched_requests_queued"] == 0
        assert vals["sched_engine_prefill_tokens_total"] > 0
        r = requests.post(f"http://127.0.0.1:{port}/generate", json={"sampling_params": {}}, timeout=5)
        assert r.status_code == 400
        server.should_exit = True
        th.join(10)
    finally:
        srv.stop()


def test_tensor_parallel_server_keeps_ranks_in_lockstep():
    """Rank 0 serves and broadcasts each round's admissions; followers add
    the same requests and step: every rank takes the same number of steps
    and finishes the same requests with the same tokens; a request rank 0
    refuses is never sent."""
    import os
    import subprocess
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    worker = os.path.join(root, "tests", "workers", "tp_server_worker.py")
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    procs = [subprocess.Popen([sys.executable, worker], stdout=subprocess.PIPE, stderr=subprocess.PIPE, text=True,
                              env={**os.environ, "RANK": str(r), "WORLD_SIZE": "3", "MASTER_ADDR": "127.0.0.1",
                                   "MASTER_PORT": str(port), "CUDA_VISIBLE_DEVICES": ""}) for r in range(3)]
    outs = []
    for p in procs:
        so, se = p.communicate(timeout=120)
        assert p.returncode == 0, se[-2000:]
        outs.append(json.loads([l for l in so.splitlines() if l.startswith("SRVJSON ")][0][len("SRVJSON "):]))
    r0 = outs[0]
    assert r0["error"] is None and r0["bad_rejected"] and r0["long_cancelled"]
    assert len(r0["outputs"]) == 12
    assert all(o["idle"] for o in outs)  # the cancelled request left no pages behind on any rank
    for o in outs[1:]:
        assert o["steps"] == r0["steps"] > 0
        assert o["finished"] == r0["finished"]
    assert [r0["outputs"][str(i)] for i in range(12)] == [r0["finished"][str(i)] for i in range(12)]


def test_tensor_parallel_server_fails_requests_when_a_rank_leaves():
    """A follower leaves between rounds: rank 0's server fails its pending
    requests (rank failure or the group's timeout) within seconds instead of
    waiting for ever, and the surviving follower ends too."""
    import os
    import subprocess
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    worker = os.path.join(root, "tests", "workers", "tp_server_worker.py")
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    procs = [subprocess.Popen([sys.executable, worker, "leave"], stdout=subprocess.PIPE, stderr=subprocess.PIPE,
                              text=True, env={**os.environ, "RANK": str(r), "WORLD_SIZE": "3",
                                              "MASTER_ADDR": "127.0.0.1", "MASTER_PORT": str(port),
                                              "CUDA_VISIBLE_DEVICES": ""}) for r in range(3)]
    outs = {}
    for r, p in enumerate(procs):
        so, se = p.communicate(timeout=120)
        lines = [l for l in so.splitlines() if l.startswith("SRVJSON ")]
        assert lines, (r, se[-2000:])
        outs[r] = json.loads(lines[0][len("SRVJSON "):])
    assert outs[2]["left"]
    assert all(e is not None for e in outs[0]["failed"]), outs[0]
    assert outs[0]["elapsed"] < 30, outs[0]
    # the survivor ends with the heartbeat's RankFailure or the group's own error
    # (timeout or a closed connection, depending on which is seen first)
    f = outs[1]["follower"]
    assert f == "RankFailure" or f.endswith("Error"), outs[1]


def test_serving_ab_interleaves_arms_and_restores_env():
    """The A/B driver builds one engine per (round, arm) with the arm's
    engine options and SCHED_* variables, interleaves the arms round by
    round, restores the environment, and keeps each arm's best round."""
    import os

    from sched_pass_b200.benchmarks.serving_ab import run_ab
    seen = []

    def make(kw):
        seen.append((kw.get("levers"), os.environ.get("SCHED_ENFORCE")))
        return FakeEngine()

    before = os.environ.get("SCHED_ENFORCE")
    work = loadgen.dispersed(12, mu=3.0, sigma=0.5, lo=4, hi=40, out=3, vocab=1000, seed=3, rate=100.0)
    lines = []
    best = run_ab(make, work, ["stock", "observe", "enforce"], 2, emit=lines.append)
    assert seen == [(False, before), (True, "0"), (True, "1")] * 2
    assert os.environ.get("SCHED_ENFORCE") == before
    assert set(best) == {"stock", "observe", "enforce"} and all(b["n_ok"] == 12 for b in best.values())
    assert [json.loads(l).get("arm") for l in lines[:-1]] == ["stock", "observe", "enforce"] * 2
    assert "summary" in json.loads(lines[-1])


def test_cancel_running_and_queued_requests():
    """A running request and one cancelled right after submission both end
    with CancelledError; their pages return to the pool and the server keeps
    serving; an unknown name is refused."""
    import concurrent.futures as cf

    import pytest
    class SlowFake(FakeEngine):
        def step(self):
            time.sleep(0.001)  # a long request stays running for seconds
            return super().step()

    srv = EngineServer(SlowFake()).start()
    try:
        f = srv.submit([1, 2, 3], 4000, name="long")
        for _ in range(500):
            if srv._pending:
                break
            time.sleep(0.01)
        srv.cancel("long")
        with pytest.raises(cf.CancelledError):
            f.result(timeout=10)
        g = srv.submit([4, 5], 4000, name="q")
        srv.cancel("q")
        with pytest.raises(cf.CancelledError):
            g.result(timeout=10)
        assert srv.submit([7], 2).result(timeout=10)["output_ids"] == [8, 9]
        for _ in range(500):
            if srv.engine.sched.idle:
                break
            time.sleep(0.01)
        sched = srv.engine.sched
        assert sched.idle and sched.alloc.free == sched.alloc.num_pages
        with pytest.raises(KeyError):
            srv.cancel("nope")
    finally:
        srv.stop()


def test_streaming_tokens_in_process_and_over_http():
    """Tokens stream as the engine produces them: the in-process queue and
    the server-sent events carry exactly the final output, in order."""
    srv = EngineServer(FakeEngine()).start()
    try:
        f = srv.submit(list(range(30)), 6, stream=True)
        got = []
        while True:
            item = f.tokens.get(timeout=10)
            if item is None:
                break
            got.append(item)
        out = f.result(timeout=10)["output_ids"]
        assert [t for _, t in got] == out and [i for i, _ in got] == list(range(6))
        # a streamed request the engine refuses ends its stream too (no client waits for ever)
        bad = srv.submit(list(range(5000)), 2, stream=True)
        assert bad.tokens.get(timeout=10) is None and bad.exception(timeout=10) is not None

        import uvicorn
        with socket.socket() as s:
            s.bind(("127.0.0.1", 0))
            port = s.getsockname()[1]
        server = uvicorn.Server(uvicorn.Config(srv.app(), host="127.0.0.1", port=port, log_level="error"))
        th = threading.Thread(target=server.run, daemon=True)
        th.start()
        for _ in range(200):
            if server.started:
                break
            time.sleep(0.02)
        import requests
        r = requests.post(f"http://127.0.0.1:{port}/generate", json={"input_ids": [3, 4, 5], "stream": True,
                                                                     "sampling_params": {"max_new_tokens": 4}},
                          stream=True, timeout=10)
        events = [json.loads(l[len("data: "):]) for l in r.iter_lines(decode_unicode=True) if l.startswith("data: ")]
        assert [e["token"] for e in events[:-1]] == [6, 7, 8, 9]
        assert events[-1]["done"] and events[-1]["meta_info"]["completion_tokens"] == 4
        server.should_exit = True
        th.join(10)
    finally:
        srv.stop()


def test_engine_error_fails_admitted_queued_and_later_requests():
    """When a step raises, the running request, a request still in the
    inbox and a request submitted afterwards all fail, and every stream
    ends: no caller waits for ever."""
    import concurrent.futures as cf

    import pytest

    gate = threading.Event()

    class Broken(FakeEngine):
        def step(self):
            gate.wait(10)  # hold the first step until the second request is queued
            raise RuntimeError("injected step failure")

    srv = EngineServer(Broken()).start()
    try:
        a = srv.submit([1, 2, 3], 4, stream=True)
        for _ in range(500):
            if srv._pending:
                break
            time.sleep(0.01)
        b = srv.submit([4, 5], 4, stream=True)  # queued behind the failing step
        gate.set()
        for f in (a, b):
            with pytest.raises(RuntimeError, match="injected"):
                f.result(timeout=10)
            assert f.tokens.get(timeout=10) is None
        c = srv.submit([6], 2, stream=True)
        with pytest.raises(RuntimeError, match="engine stopped"):
            c.result(timeout=10)
        assert c.tokens.get(timeout=10) is None
        assert isinstance(srv.error, RuntimeError)
    finally:
        srv.stop()
