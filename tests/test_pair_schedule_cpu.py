"""The CTA-pair GEMM's schedule restated on the host (ops/pair_schedule.py):
the plans the B200 reported for measured shapes, and the invariants the
kernel relies on, over a sweep of shapes."""
import itertools

import numpy as np
import pytest

from sched_pass_b200.ops import pair_schedule as ps

CAP = 74  # resident two-CTA clusters of the pair kernel on a 148-SM B200


@pytest.mark.parametrize("shape,want", [
    # (T, N, K), (clusters, whole tiles, k-ranges) as sched_gemm_pair_plan reported on a B200
    ((256, 6144, 4096), (72, 0, 3)),
    ((1536, 4096, 4096), (74, 74, 3)),
    ((512, 28672, 4096), (74, 222, 8)),
    ((1536, 4096, 14336), (74, 74, 3)),
])
def test_plans_reported_on_b200(shape, want):
    pl = ps.plan(*shape, CAP)
    assert (pl.np, pl.whole, pl.splits) == want
    whole = ps.plan(*shape, CAP, may_split=False)
    assert whole.splits == 1 and whole.whole == ps.tiles_of(shape[0], shape[1])


def test_single_cta_shapes_and_switches():
    assert ps.plan(16, 4096, 4096, CAP).np == 0           # decode sizes stay single-CTA
    assert ps.plan(300, 4096 + 128, 4096, CAP).np == 0    # N not a multiple of 256
    assert ps.plan(1536, 4096, 4096, CAP, mode=0).np == 0  # SCHED_GEMM_PAIR=0
    assert ps.plan(16, 4096, 4096, CAP, mode=1).np > 0     # =1: every eligible shape
    assert ps.plan(1536, 4096, 4096, CAP, default_grid=False).np == 0
    # qkv at T=1536: 144 tiles, 70 in the last wave: one k-range each fits, so no split
    assert ps.plan(1536, 6144, 4096, CAP).splits == 1


def test_scratch_limits_the_split():
    T, N, K = 512, 4096, 4096  # 32 tiles, 2 k-ranges each: exactly 2^22 floats of partials
    assert ps.scratch(T, N, ps.plan(T, N, K, CAP, ws_floats=1 << 22, counters=1 << 14))[0] == 1 << 22
    assert ps.plan(T, N, K, CAP, ws_floats=(1 << 22) - 1).splits == 1
    assert ps.plan(T, N, K, CAP, counters=127).splits == 1
    assert ps.plan(T, N, K, CAP, ws_floats=0).splits == 1


SHAPES = list(itertools.product([256, 300, 512, 777, 1536, 2048], [4096, 6144, 28672], [4096, 14336]))


@pytest.mark.parametrize("T,N,K", SHAPES)
def test_schedule_invariants(T, N, K):
    pl = ps.plan(T, N, K, CAP)
    if pl.np == 0:
        return
    tiles, kb = ps.tiles_of(T, N), K // ps.BK
    assert 0 < pl.np <= CAP and 1 <= pl.splits <= ps.MAX_SPLITS
    ws, cnt = ps.scratch(T, N, pl)
    assert ws <= 1 << 24 and cnt <= 1 << 16
    covered = np.zeros((tiles, kb), dtype=np.int32)
    per_cluster = ps.cluster_units(T, N, K, pl)
    for units in per_cluster:
        ksplit = [i for i, u in enumerate(units) if u[3] >= 0]
        # at most one k-range unit per cluster, and it is the cluster's first:
        # so the k-ranges of a tile are co-resident in a launch that fits
        assert ksplit in ([], [0])
        for tile, k0, k1, _ in units:
            assert k1 - k0 >= (ps.MIN_SPLIT_KB if pl.splits > 1 and k1 - k0 < kb else 1)
            covered[tile, k0:k1] += 1
    assert (covered == 1).all(), "every k-block of every tile exactly once"
    # the k-ranges of a split tile sum slab slices that partition its slabs
    for tile in range(pl.whole, tiles):
        t0 = (tile % ((T + ps.TN - 1) // ps.TN)) * ps.TN
        nch = min(ps.TN, T - t0 + ps.SLAB - 1) // ps.SLAB
        got = []
        for s in range(pl.splits):
            c0, c1 = ps.slab_slice(s, pl.splits, T, tile, N)
            got.extend(range(c0, c1))
        assert got == list(range(nch))
    # the makespan in whole-tile times beats whole tiles on the same clusters
    if pl.splits > 1:
        waves_whole = -(-tiles // CAP)
        assert pl.whole // CAP + 1 / pl.splits < waves_whole


def test_slices_sum_in_split_order_whatever_the_arrival():
    """Each k-range writes its partial to its own slot; once all have
    arrived, each sums its slab slice over the slots in split order. The
    output is then the same bits for every arrival order, which a sum in
    arrival order would not be (fp32 addition is not associative)."""
    rng = np.random.default_rng(0)
    S, nch = 5, 16
    parts = (rng.standard_normal((S, nch, 64)) * 10.0 ** rng.integers(-3, 4, (S, 1, 1))).astype(np.float32)

    def run(arrival):
        slots = [None] * S
        for s in arrival:
            slots[s] = parts[s]
        out = np.empty((nch, 64), np.float32)
        for s in arrival:
            c0, c1 = s * nch // S, (s + 1) * nch // S
            acc = slots[0][c0:c1].copy()
            for s2 in range(1, S):
                acc = acc + slots[s2][c0:c1]
            out[c0:c1] = acc
        return out

    perms = list(itertools.permutations(range(S)))
    ref = run(range(S))
    assert all(np.array_equal(run(a), ref) for a in perms)
    by_arrival = []
    for a in perms:
        acc = parts[a[0]].copy()
        for s in a[1:]:
            acc = acc + parts[s]
        by_arrival.append(acc)
    assert any(not np.array_equal(b, by_arrival[0]) for b in by_arrival)
