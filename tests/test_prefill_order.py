"""pi for prefill attention tiles on the host: LPT by causal work is a
permutation of the plan's tiles, longest first, stable on ties; identity
keeps the plan. (The kernel's tiles are independent, so any order gives the
same bits: checked on GPUs by the engine tests.)"""
import random

import pytest

from sched_pass_b200.engine.engine import order_prefill_tiles


def test_lpt_is_a_stable_longest_first_permutation():
    rng = random.Random(0)
    tiles = [(rng.randrange(8), 64 * i, rng.choice([64, 64, 64, 17]), rng.randrange(0, 4096, 16)) for i in range(40)]
    out = order_prefill_tiles(tiles, "lpt")
    assert sorted(out) == sorted(tiles)
    cost = [t[2] * (t[3] + t[2]) for t in out]
    assert cost == sorted(cost, reverse=True)
    for a, b in zip(out, out[1:]):  # ties keep plan order
        if a[2] * (a[3] + a[2]) == b[2] * (b[3] + b[2]):
            assert tiles.index(a) < tiles.index(b)
    assert order_prefill_tiles(tiles, "identity") == tiles
    # a causal prompt's later tiles carry more keys: they go first
    one = [(0, 64 * i, 64, 64 * i) for i in range(24)]
    assert [t[1] for t in order_prefill_tiles(one)] == [64 * i for i in range(23, -1, -1)]
    with pytest.raises(ValueError):
        order_prefill_tiles(tiles, "random")
