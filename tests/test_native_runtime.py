"""Native host runtime: page allocator, decode planner, orders (GPU-free)."""
import numpy as np
import pytest
import torch

from sched_pass_b200.engine import native
from sched_pass_b200.runtime.sched_rt import SchedPlane


def test_allocator_all_or_nothing_and_double_free():
    a = native.PageAllocator(8)
    p = a.take(5)
    assert p is not None and len(set(p.tolist())) == 5 and a.free == 3
    assert a.take(4) is None and a.free == 3
    a.give(p[:2])
    with pytest.raises(ValueError):
        a.give(p[:1])
    assert a.free == 5


def test_plan_decode_covers_every_token_once():
    rng = np.random.default_rng(0)
    lens = rng.integers(1, 3000, size=37).astype(np.int32)
    for S in (1, 2, 3, 8):
        items, mreq, mbeg = native.plan_decode(lens, S)
        assert items.shape == (37 * S, 4)
        cover = np.zeros((37, 3100), dtype=np.int32)
        for b, lo, hi, part in items:
            assert lo % 128 == 0 and hi >= lo
            cover[b, lo:hi] += 1
            assert (part == -1) == (S == 1)
        for b in range(37):
            assert (cover[b, :lens[b]] == 1).all() and cover[b, lens[b]:].sum() == 0
        if S > 1:
            assert (mbeg == np.arange(38) * S).all() and (mreq == np.arange(37)).all()


@pytest.mark.parametrize("block", [1, 4, 16])
def test_native_orders_match_python_plane(block):
    rng = np.random.default_rng(block)
    cost = rng.integers(1, 50, size=203).astype(np.float32)
    ref = SchedPlane._grouped_lpt(torch.from_numpy(cost), block).numpy()
    assert (native.grouped_lpt(cost, block) == ref).all()
    R = 64
    ref_r = SchedPlane.region_order(torch.from_numpy(cost), R, block).numpy()
    got_r = native.region_order(cost, R, block)
    assert (got_r == ref_r).all()
    assert sorted(got_r.tolist()) == list(range(203))


def test_task_costs():
    items = np.array([[0, 0, 256, -1], [1, 0, 10, -1]], dtype=np.int32)
    c = native.task_costs(items, 2, 3)
    assert c.tolist() == [256.0] * 3 + [10.0] * 3
