"""The fused GEMM + all-reduce protocol, emulated among gloo ranks on the
CPU (sched_pass_b200/parallel/protocol.py): the flag counts of cluster
split-K agree with the publishers, results are bit-identical to the
kernel's rank-order reduction and close to the fp32 sum, a slow rank is
tolerated because two buffer sets alternate (one set is not enough), and a
lost push ends in a peer-timeout status instead of a hang. The same for the
decode-size line exchange, with per-peer and with multicast writes, and
with lines whose 8-byte halves land separately."""
import json
import os
import shutil
import socket
import subprocess
import sys
import tempfile

import numpy as np
import pytest
import torch

from sched_pass_b200.parallel import protocol as P

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
WORKER = os.path.join(ROOT, "tests", "workers", "protocol_worker.py")


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def launch(scenario, world, timeout=120):
    d = tempfile.mkdtemp(prefix="sched_proto_")
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
                if line.startswith("PROTOJSON "):
                    outs[r] = json.loads(line[len("PROTOJSON "):])
        return outs
    finally:
        shutil.rmtree(d, ignore_errors=True)


@pytest.mark.parametrize("TN", [16, 32, 64, 128])
def test_chunk_contributors_match_the_publishers(TN):
    """gemm.cu computes the readers' count (chunk_contributors) and the
    publishers' releases (publish_rows) separately; they must agree for
    every tile fill and cluster size, or a reader waits forever."""
    for cs in range(1, 9):
        for tv in range(1, TN + 1):
            got = np.zeros(TN // P.KSLAB, dtype=int)
            for r in range(cs):
                lo, hi = P.share_bounds(tv, cs, r) if cs > 1 else (0, tv)
                for ch in P.published_chunks(lo, hi):
                    got[ch] += 1
            for ch in range(TN // P.KSLAB):
                want = P.chunk_contributors(tv, cs, ch) if ch * P.KSLAB < tv else 0
                assert got[ch] == want, (TN, cs, tv, ch)


def test_reduce_rank_order_is_sequential_fp32():
    parts = P.to_bf16_bits(torch.tensor([[1.0, 3.0, 1.0 + 2.0 ** -7],
                                         [2.0 ** -9, -3.0, 2.0 ** -8],
                                         [2.0 ** -9, 1.0, 0.0]]))[:, None, :]
    got = P.from_bf16_bits(P.reduce_rank_order(parts))
    # (1 + 2^-9) + 2^-9 = 1 + 2^-8 in fp32: a tie between bf16 neighbours, rounds to even (1.0);
    # (3 - 3) + 1 = 1; 1 + 3 * 2^-8: a tie, rounds to even (1 + 2^-6)
    assert got.tolist() == [[1.0, 1.0, 1.0 + 2.0 ** -6]]


@pytest.mark.parametrize("world", [2, 3])
def test_emulated_allreduce_is_exact(world):
    outs = launch("exact", world)
    for r in range(world):
        assert outs[r]["bad"] == [], outs[r]
        assert set(outs[r]["statuses"]) == {P.STATUS_OK}


def test_slow_rank_is_safe_with_two_sets():
    outs = launch("skew", 2)
    for r in (0, 1):
        assert outs[r]["wrong"] == 0 and set(outs[r]["statuses"]) == {P.STATUS_OK}, outs[r]


def test_one_set_breaks_under_a_slow_rank():
    outs = launch("oneset", 2)
    # the fast rank's next push lands in the slow rank's slab before it reduced
    assert outs[1]["wrong"] > 0 or P.STATUS_PEER_TIMEOUT in outs[1]["statuses"], outs


def test_lost_push_times_out_with_status():
    outs = launch("drop", 2)
    for r in (0, 1):
        assert outs[r]["status"] == P.STATUS_PEER_TIMEOUT and outs[r]["elapsed"] < 10, outs[r]


@pytest.mark.parametrize("world", [2, 3])
@pytest.mark.parametrize("scen", ["ll_exact", "ll_torn"])
def test_line_exchange_is_exact(world, scen):
    """Epoch-tagged lines, written per peer or through multicast (each
    8-byte half reaching every copy at once), and with every first half
    landing before any second half: every rank's output is the kernel's
    rank-order reduction, bit for bit, with no timeout."""
    outs = launch(scen, world)
    for r in range(world):
        assert outs[r]["bad"] == [], outs[r]
        assert set(outs[r]["statuses"]) == {P.STATUS_OK}
        assert outs[r]["state"] == outs[r]["calls"]  # the epoch advanced once per call


def test_line_exchange_tolerates_a_slow_rank():
    """A rank that pushes late: the others poll their own copies until the
    late lines carry the call's epoch, and never take the same set's lines
    from two calls before (their epoch differs)."""
    outs = launch("ll_skew", 2)
    for r in (0, 1):
        assert outs[r]["bad"] == [] and set(outs[r]["statuses"]) == {P.STATUS_OK}, outs[r]


def test_line_exchange_lost_row_times_out_with_status():
    outs = launch("ll_drop", 2)
    for r in (0, 1):
        assert outs[r]["status"] == P.STATUS_PEER_TIMEOUT and outs[r]["elapsed"] < 10, outs[r]


def test_epoch_state_skips_zero():
    assert P.state_after_call(7) == 7
    assert P.state_after_call(0xFFFFFFFF) == 1  # next call uses epoch 2: never 0
