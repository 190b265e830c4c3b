"""Host-side model of the CTA-pair GEMM's schedule (``gemm_pair_kernel``,
``pair_plan_epi`` and ``pair_unit`` in csrc/kernels/gemm.cu).

A launch of ``np`` clusters (two CTAs each) covers ``tiles`` output tiles of
256 weight rows x 256 tokens. The tiles of the full waves run whole; each
tile of the last, partly filled wave runs as ``splits`` k-ranges. Units go
to clusters round-robin, k-range units first, so each k-range unit is the
first unit of its cluster. After every k-range of a tile has written its
fp32 partial, k-range ``s`` sums the tile's token slabs ``[s * nch / splits,
(s + 1) * nch / splits)`` over all partials in split order.

The functions here restate that arithmetic so that its invariants can be
checked without a GPU (every k-block of every tile computed once, no cluster
holding two k-range units, slab slices that partition the tile, scratch
within the caller's workspace) and a call's plan predicted from its shape
and the GPU's cluster capacity.
"""
from __future__ import annotations

from dataclasses import dataclass

TN = 256            # tokens per pair tile
BM = 128            # weight rows per CTA (a pair tile has 2 * BM)
BK = 64             # k-block
SLAB = 16           # tokens per epilogue slab
MAX_SPLITS = 8      # k-ranges per tile of the last wave, at most
MIN_SPLIT_KB = 8    # k-blocks per k-range, at least
PART_FLOATS = TN * BM  # one CTA's fp32 partial of a tile


@dataclass(frozen=True)
class PairPlan:
    np: int = 0      # clusters launched (0: the single-CTA schedules run instead)
    whole: int = 0   # tiles [0, whole) run whole
    splits: int = 1  # k-ranges per tile of [whole, tiles)


def tiles_of(T: int, N: int) -> int:
    return (N // (2 * BM)) * ((T + TN - 1) // TN)


def plan(T: int, N: int, K: int, cap: int, ws_floats: int = 1 << 24, counters: int = 1 << 16, *,
         mode: int = -1, may_split: bool = True, default_grid: bool = True) -> PairPlan:
    """The launch ``sched_gemm_run`` makes for a store / SwiGLU / RoPE+KV call
    of this shape on a GPU with ``cap`` resident clusters of two pair CTAs.
    ``mode``: ``SCHED_GEMM_PAIR`` (-1 unset, 0 off, 1 every eligible shape);
    ``may_split``: ``SCHED_GEMM_PAIR_SPLIT`` != 0."""
    if mode == 0 or not default_grid or N % (2 * BM) or K % BK:
        return PairPlan()
    if T < (1 if mode == 1 else 256) or cap <= 0:
        return PairPlan()
    tiles = tiles_of(T, N)
    full, rem = divmod(tiles, cap)
    kb = K // BK
    S = 1
    if may_split and rem > 0:
        S = min(cap // rem, kb // MIN_SPLIT_KB, MAX_SPLITS)
        need = rem * S * 2 * PART_FLOATS
        if S < 2 or need > ws_floats or 4 * rem > counters:
            S = 1
    if S > 1:
        pl = PairPlan(np=cap if full > 0 else rem * S, whole=full * cap, splits=S)
        waves = full + 1.0 / S
    else:
        pl = PairPlan(np=min(cap, tiles), whole=tiles, splits=1)
        waves = float((tiles + cap - 1) // cap)
    busy = tiles / (waves * cap)
    return pl if (mode == 1 or busy >= 0.3) else PairPlan()


def n_units(tiles: int, pl: PairPlan) -> int:
    return pl.whole + (tiles - pl.whole) * pl.splits if pl.splits > 1 else tiles


def unit(pl: PairPlan, tiles: int, u: int, kb: int) -> tuple[int, int, int, int]:
    """(tile, first k-block, end k-block, k-range index or -1) of unit u."""
    if pl.splits <= 1:
        return u, 0, kb, -1
    nsplit = (tiles - pl.whole) * pl.splits
    if u >= nsplit:
        return u - nsplit, 0, kb, -1
    s = u % pl.splits
    return pl.whole + u // pl.splits, s * kb // pl.splits, (s + 1) * kb // pl.splits, s


def cluster_units(T: int, N: int, K: int, pl: PairPlan) -> list[list[tuple[int, int, int, int]]]:
    """The units each cluster runs, in order."""
    tiles, kb = tiles_of(T, N), K // BK
    out = [[] for _ in range(pl.np)]
    for u in range(n_units(tiles, pl)):
        out[u % pl.np].append(unit(pl, tiles, u, kb))
    return out


def slab_slice(split: int, splits: int, T: int, tile: int, N: int) -> tuple[int, int]:
    """Token slabs [c0, c1) of a split tile that k-range ``split`` sums."""
    t_tiles = (T + TN - 1) // TN
    t0 = (tile % t_tiles) * TN
    nch = min(TN, T - t0 + SLAB - 1) // SLAB
    return split * nch // splits, (split + 1) * nch // splits


def scratch(T: int, N: int, pl: PairPlan) -> tuple[int, int]:
    """(workspace floats, counters) the launch uses."""
    if pl.splits <= 1:
        return 0, 0
    rem = tiles_of(T, N) - pl.whole
    return rem * pl.splits * 2 * PART_FLOATS, 4 * rem
