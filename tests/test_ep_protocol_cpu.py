"""The expert-parallel MoE exchange, emulated among gloo ranks on the CPU
(sched_pass_b200/parallel/ep_protocol.py): every rank's combined output is
exactly the routed sum over the assignments it kept, capacity drops are
accounted on the source, and a source that routes nothing to a slow owner is
safe with two alternating buffer sets but not with one."""
import json
import os
import shutil
import socket
import subprocess
import sys
import tempfile

from sched_pass_b200.parallel.protocol import STATUS_OK, STATUS_PEER_TIMEOUT

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
WORKER = os.path.join(ROOT, "tests", "workers", "ep_protocol_worker.py")


def launch(scenario, world, sets, timeout=180):
    d = tempfile.mkdtemp(prefix="sched_ep_")
    try:
        with socket.socket() as s:
            s.bind(("127.0.0.1", 0))
            port = s.getsockname()[1]
        procs = []
        for r in range(world):
            env = {**os.environ, "RANK": str(r), "WORLD_SIZE": str(world), "MASTER_ADDR": "127.0.0.1",
                   "MASTER_PORT": str(port), "CUDA_VISIBLE_DEVICES": "", "PROTO_DIR": d}
            procs.append(subprocess.Popen([sys.executable, WORKER, scenario, str(sets)], env=env,
                                          stdout=subprocess.PIPE, stderr=subprocess.PIPE, text=True))
        outs = {}
        for r, p in enumerate(procs):
            try:
                so, se = p.communicate(timeout=timeout)
            except subprocess.TimeoutExpired:
                p.kill()
                so, se = p.communicate()
                raise AssertionError(f"rank {r} hung in {scenario}: {se[-2000:]}")
            assert p.returncode == 0, se[-3000:]
            for line in so.splitlines():
                if line.startswith("EPJSON "):
                    outs[r] = json.loads(line[len("EPJSON "):])
        return outs
    finally:
        shutil.rmtree(d, ignore_errors=True)


def test_exchange_is_exact():
    outs = launch("ep_exact", 3, 2)
    for r in range(3):
        assert outs[r]["wrong"] == 0 and set(outs[r]["statuses"]) == {STATUS_OK}, outs[r]
        assert outs[r]["dropped"] == 0


def test_capacity_drops_are_zero_rows_on_the_source():
    """Slots at or above the capacity drop the assignment: its row never
    comes back and the source's combine counts on it as dropped."""
    outs = launch("ep_drops", 3, 2)
    assert sum(outs[r]["dropped"] for r in range(3)) > 0
    for r in range(3):
        assert outs[r]["wrong"] == 0 and set(outs[r]["statuses"]) == {STATUS_OK}, outs[r]


def test_two_sets_keep_a_fast_source_off_a_slow_owners_counts():
    outs = launch("ep_skew", 3, 2)
    for r in range(3):
        assert outs[r]["wrong"] == 0 and set(outs[r]["statuses"]) == {STATUS_OK}, outs[r]


def test_one_set_breaks_when_a_source_skips_a_slow_owner():
    """Rank 0 routes nothing to rank 2, which is slow: rank 0 finishes each
    layer without waiting for rank 2 and its next dispatch reaches rank 2's
    counts before rank 2 clears them for the previous layer."""
    outs = launch("ep_skew", 3, 1)
    assert any(outs[r]["wrong"] or STATUS_PEER_TIMEOUT in outs[r]["statuses"] for r in range(3)), outs
