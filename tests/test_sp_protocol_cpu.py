"""The sequence-parallel protocol (reduce-scatter GEMM epilogue -> owner's
reduce + residual + RMSNorm + all-gather push -> ready-gated GEMM),
emulated among gloo ranks on the CPU (sched_pass_b200/parallel/sp_protocol.py):
row ownership partitions the tokens, the owner's reduction is bit-identical to
the fused all-reduce's, every rank gathers the same rows, alternating sets
survive a slow rank and token counts that shrink and grow, and a lost push
ends in a peer-timeout status instead of a hang."""
import json
import os
import shutil
import socket
import subprocess
import sys
import tempfile

import pytest

from sched_pass_b200.parallel import protocol as P
from sched_pass_b200.parallel.sp import owned_rows, row_owner

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
WORKER = os.path.join(ROOT, "tests", "workers", "sp_protocol_worker.py")


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def launch(scenario, world, timeout=180):
    d = tempfile.mkdtemp(prefix="sched_sp_")
    try:
        port = _port()
        procs = []
        for r in range(world):
            env = {**os.environ, "RANK": str(r), "WORLD_SIZE": str(world), "MASTER_ADDR": "127.0.0.1",
                   "MASTER_PORT": str(port), "CUDA_VISIBLE_DEVICES": "", "PROTO_DIR": d}
            procs.append(subprocess.Popen([sys.executable, WORKER, scenario], env=env, stdout=subprocess.PIPE,
                                          stderr=subprocess.PIPE, text=True))
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
                if line.startswith("SPJSON "):
                    outs[r] = json.loads(line[len("SPJSON "):])
        return outs
    finally:
        shutil.rmtree(d, ignore_errors=True)


def test_row_ownership_partitions_the_tokens():
    """sp_row_owner and sp_row_begin (gemm_api.h) are computed separately by
    the pushing GEMM and the reducing norm; they must agree, or a row is
    reduced twice or waited for forever."""
    for world in range(1, 9):
        for T in range(1, 300):
            seen = []
            for r in range(world):
                lo, hi = owned_rows(r, world, T)
                assert 0 <= lo <= hi <= T
                for t in range(lo, hi):
                    assert row_owner(t, world, T) == r, (world, T, t)
                seen += range(lo, hi)
            assert seen == list(range(T)), (world, T)


@pytest.mark.parametrize("world", [2, 3, 5])
def test_emulated_sequence_parallel_is_exact(world):
    outs = launch("exact", world)
    for r in range(world):
        assert outs[r]["bad"] == [], outs[r]
        assert set(outs[r]["statuses"]) == {P.STATUS_OK}, outs[r]


def test_slow_rank_is_safe():
    outs = launch("skew", 2)
    for r in (0, 1):
        assert outs[r]["bad"] == [] and set(outs[r]["statuses"]) == {P.STATUS_OK}, outs[r]


def test_lost_push_times_out_with_status():
    outs = launch("drop", 2)
    # the owner of row 0 (rank 0) never gets the dropped tile; every rank's
    # consumer then misses that row's ready flag
    assert outs[0]["status"] == P.STATUS_PEER_TIMEOUT, outs
    for r in (0, 1):
        assert outs[r]["consume"] == P.STATUS_OK or outs[r]["consume"] == P.STATUS_PEER_TIMEOUT
        assert outs[r]["elapsed"] < 10, outs[r]
