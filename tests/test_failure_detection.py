"""Failure detection among CPU (gloo) ranks: a rank that dies, one that
leaves, a dropped message and a collective with a missing peer all end in a
bounded time with a clear error on the survivors. No GPU is involved."""
import json
import os
import socket
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
WORKER = os.path.join(ROOT, "tests", "workers", "fault_worker.py")


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def launch(scenario, world, timeout=60):
    port = _port()
    procs = []
    for r in range(world):
        env = {**os.environ, "RANK": str(r), "WORLD_SIZE": str(world), "MASTER_ADDR": "127.0.0.1",
               "MASTER_PORT": str(port), "CUDA_VISIBLE_DEVICES": ""}
        procs.append(subprocess.Popen([sys.executable, WORKER, scenario], env=env, stdout=subprocess.PIPE,
                                      stderr=subprocess.PIPE, text=True))
    outs = {}
    codes = {}
    for r, p in enumerate(procs):
        try:
            so, se = p.communicate(timeout=timeout)
        except subprocess.TimeoutExpired:
            p.kill()
            so, se = p.communicate()
            raise AssertionError(f"rank {r} hung in scenario {scenario}: {se[-2000:]}")
        codes[r] = p.returncode
        for line in so.splitlines():
            if line.startswith("FAULTJSON "):
                outs[r] = json.loads(line[len("FAULTJSON "):])
    return outs, codes


def test_crashed_rank_is_detected_by_survivors():
    outs, codes = launch("crash", 3)
    assert codes[2] == 3
    for r in (0, 1):
        assert outs[r].get("failure") == [2] or "error" in outs[r], outs[r]
        assert outs[r]["elapsed"] < 20


def test_graceful_leave_is_seen_at_once():
    outs, codes = launch("leave", 2)
    assert outs[1].get("left")
    assert outs[0].get("failure") == [1], outs[0]


def test_dropped_flag_times_out_instead_of_hanging():
    outs, _ = launch("dropflag", 2)
    assert outs[0]["got"] is False and outs[0]["elapsed"] < 5
    assert outs[1]["got"] is True


def test_collective_with_missing_peer_errors_out():
    outs, _ = launch("collective", 2)
    assert "error" in outs[0] or "failure" in outs[0], outs[0]
    assert outs[1].get("ok")


def test_rank_that_never_joins_fails_the_rendezvous():
    code = (
        "import datetime, sys, torch.distributed as dist\n"
        "try:\n"
        "    dist.init_process_group('gloo', init_method='tcp://127.0.0.1:%d', rank=0, world_size=2,\n"
        "                            timeout=datetime.timedelta(seconds=3))\n"
        "    print('JOINED')\n"
        "except Exception as e:\n"
        "    print('REFUSED', type(e).__name__)\n" % _port())
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=60,
                       env={**os.environ, "CUDA_VISIBLE_DEVICES": ""})
    assert "REFUSED" in r.stdout, r.stdout + r.stderr
