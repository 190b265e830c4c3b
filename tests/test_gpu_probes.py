"""The lever probes: every acquisition mode runs each task exactly once, and
the cache-policy stream reads at a sane fraction of HBM bandwidth."""
import numpy as np
import pytest
import torch

from sched_pass_b200 import ops
from sched_pass_b200._ext import ext

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("mode", [0, 1, 2])
@pytest.mark.parametrize("memory", [False, True])
def test_task_probe_exactly_once(mode, memory):
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    R = ext().probe_tasks_occupancy() * sms
    n = 3 * R + 17
    rng = np.random.default_rng(mode)
    cost = rng.integers(1000, 20000, size=n) if not memory else np.full(n, 4096)
    c = torch.from_numpy(cost.astype(np.int32)).cuda()
    hits = torch.zeros(n, dtype=torch.int32, device="cuda")
    per = torch.zeros(max(n, R), dtype=torch.int32, device="cuda")
    ticket = torch.zeros(1, dtype=torch.int32, device="cuda")
    sink = torch.zeros(4, dtype=torch.int32, device="cuda")
    data = torch.zeros(1 << 22, dtype=torch.int32, device="cuda")
    ext().probe_tasks(c, mode, R, int(memory), data, hits, per, ticket, sink, ops.status_buffer())
    torch.cuda.synchronize()
    ops.check_status()
    assert (hits == 1).all()
    assert int(per.sum()) == n


def test_stream_probe_policies():
    src = torch.zeros(1 << 28, dtype=torch.int32, device="cuda")  # 1 GiB
    sink = torch.zeros(1 << 12, dtype=torch.int32, device="cuda")
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    for pol in range(5):
        ext().probe_stream(src, pol, sink, sms * 4)
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        ext().probe_stream(src, pol, sink, sms * 4)
        b.record()
        b.synchronize()
        gbs = src.numel() * 4 / a.elapsed_time(b) / 1e6
        assert gbs > 1000, (pol, gbs)


def test_pdl_pairs_bit_exact():
    """Programmatic dependent launch changes timing, never results: the
    consumer reads the producer's output after griddepcontrol.wait."""
    n = 1 << 20
    buf = torch.zeros(n, device="cuda")
    table = torch.rand(256, device="cuda")
    outs = []
    for pdl in (False, True):
        for prologue in (0, 64):
            out = torch.zeros(n, device="cuda")
            buf.zero_()
            ext().probe_pdl_pairs(buf, out, table, 512, prologue, pdl, 3)
            torch.cuda.synchronize()
            outs.append(out)
            if prologue == 0:
                assert torch.equal(out, buf * 2) and buf.abs().sum().item() > 0
    assert torch.equal(outs[0], outs[2]) and torch.equal(outs[1], outs[3])


@pytest.mark.parametrize("mode", [0, 1, 2])
def test_mix_probe_runs(mode):
    R = torch.zeros(8 << 20, dtype=torch.int32, device="cuda")   # 32 MiB reused
    S = torch.zeros(64 << 20, dtype=torch.int32, device="cuda")  # 256 MiB streamed
    sink = torch.zeros(1 << 12, dtype=torch.int32, device="cuda")
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    ext().probe_mix(R, S, mode, 0.5 if mode else 1.0, sink, sms * 4)
    torch.cuda.synchronize()
    with pytest.raises(RuntimeError):
        ext().probe_mix(R, S, 1, 0.0, sink, sms * 4)  # fraction outside (0, 1]


def test_clc_terminal_failure_rule_and_exactly_once():
    """Cluster launch control, one CTA per task, late-bound claims: every
    task runs exactly once, every worker (a CTA that launched) ends with
    exactly one failed claim and no failure before it, claimed ids are
    unique, and successes = tasks - workers (each worker ran its own task
    first); the same holds with the claim issued ahead of the body."""
    import numpy as np

    from sched_pass_b200.benchmarks import probes
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    R = int(ext().probe_tasks_occupancy()) * sms
    n = 4 * R
    for mode in (1, 2):
        _, hits, rec, n_rec, _ = probes.run_clc(probes.clc_layout(n, 1500, "interleaved"), mode, R, max_rec=64)
        assert (hits == 1).all(), mode
        claims = probes.clc_claims(rec, n_rec)
        assert (n_rec <= 64).all()
        fails = [[x for _, x in cl].count(0xFFFFFFFF) for cl in claims.values()]
        assert set(fails) == {1}, (mode, set(fails))
        assert all(cl[-1][1] == 0xFFFFFFFF for cl in claims.values())
        got = [x for cl in claims.values() for _, x in cl if x != 0xFFFFFFFF]
        assert len(got) == len(set(got)) == n - len(claims), (mode, len(got), len(claims))
        assert len(claims) <= n and len(claims) >= min(n, R // 2)


def test_clc_contract_under_shapes_participation_clusters_and_graphs():
    """CLC on B200 under the launch shapes the reference probes
    (experiments/clc/FINDINGS.md:441-802): in every case each task runs
    exactly once; with full participation the claimed CTAs are exactly the
    suffix [R, n) of the linear CTA order (2-D / 3-D ids map back linearly,
    the answer's fourth word stays zero), every worker ends with one failed
    claim, clustered launches claim whole aligned clusters, and CUDA-graph
    replays keep the same contract; with partial participation no task is
    lost or run twice."""
    from sched_pass_b200.benchmarks import probes
    rows = {r["case"]: r for r in probes.clc_shapes()}
    for name, r in rows.items():
        assert r["exactly_once"] and r["duplicate_claims"] == 0, r
    for name in ("1d", "2d_64x128", "3d_17x19x29", "cluster2", "cluster4", "graph_replay"):
        r = rows[name]
        assert r["claim_holes"] == 0 and r["claimed_max"] == r["tasks"] - 1, r
        assert r["claimed_min"] == r["launched"], r
        assert r["failures_per_worker"] == [1], r
        assert r["w_nonzero"] == 0, r
    assert rows["cluster2"]["claim_bases_aligned"] and rows["cluster4"]["claim_bases_aligned"]
    assert rows["graph_replay"]["replays_identical_contract"]
