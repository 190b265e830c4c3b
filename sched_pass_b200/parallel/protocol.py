"""CPU emulation of the fused GEMM + all-reduce peer-buffer protocol: the
oracle for the NVLink kernel and a test bed for its flag logic.

Every rank is a process (ranks meet through a gloo process group); "peer
memory" is a shared file mapping that every rank opens, the image of the
symmetric buffers the kernel reaches over NVLink. ``EmulatedAllReduce`` runs
the steps of ``csrc/kernels/gemm.cu`` (``kEpiAllReduce``: ``write_row``,
``publish_tile`` / ``publish_rows``, ``reduce_owned_chunks``) in their
order:

1. each tile's partial product is rounded to bf16 and stored into every
   rank's receive slab at ``[source rank][token][column]``;
2. the 16-token chunk flags the stored rows touch are released in every
   rank's flag array -- flag ``(source, tile, chunk)`` lives in the reader's
   array; under cluster split-K each of the ``cs`` cluster ranks adds one
   for the chunks its token share touches, and a reader waits for
   ``chunk_contributors`` of them;
3. each rank reduces the units (tile, chunk) that CTA ``u % grid`` owns: a
   bounded wait for every source's flag, the bf16 partials summed in rank
   order in fp32, rounded to bf16, the flags cleared;
4. two slab / flag sets alternate between calls, so a fast rank may run one
   call ahead of a slow one.

``reduce_rank_order`` is step 3's arithmetic on its own: given the bf16
partials the kernel left in a slab it reproduces the kernel's output bit for
bit. The reference has no collective at all (its only process group is a
world-size-1 bootstrap in test/py/test_moe_forward_gpu.py:42); this protocol
is this framework's own.
"""
from __future__ import annotations

import mmap
import os
import time

import numpy as np
import torch

KSLAB = 16          # tokens per flag chunk (gemm.cu kSlab)
BM = 128            # output columns per tile (gemm.cu BM)
STATUS_OK = 0
STATUS_PEER_TIMEOUT = 4  # common.cuh kStatusPeerTimeout


def share_bounds(tv: int, cs: int, r: int) -> tuple[int, int]:
    """Token rows [lo, hi) of a tile with ``tv`` valid rows that cluster rank
    ``r`` of ``cs`` reduces and publishes."""
    return r * tv // cs, (r + 1) * tv // cs


def published_chunks(lo: int, hi: int) -> range:
    """Chunks a publisher of rows [lo, hi) releases (gemm.cu publish_rows)."""
    if lo >= hi:
        return range(0)
    return range(lo // KSLAB, (hi - 1) // KSLAB + 1)


def chunk_contributors(tv: int, cs: int, ch: int) -> int:
    """Releases chunk ``ch`` receives from one source rank (gemm.cu
    chunk_contributors): 1 under stream-K, else the number of cluster
    shares that intersect the chunk."""
    if cs <= 1:
        return 1
    c0, c1 = ch * KSLAB, min(ch * KSLAB + KSLAB, tv)
    n = 0
    for r in range(cs):
        lo, hi = share_bounds(tv, cs, r)
        n += int(lo < hi and lo < c1 and hi > c0)
    return n


def to_bf16_bits(x: torch.Tensor) -> np.ndarray:
    """fp32 -> bf16 (round to nearest even), as uint16 bit patterns."""
    return x.to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)


def from_bf16_bits(b: np.ndarray) -> np.ndarray:
    """bf16 bit patterns -> exact fp32 values."""
    return (b.astype(np.uint32) << 16).view(np.float32)


def reduce_rank_order(partials: np.ndarray) -> np.ndarray:
    """The kernel's reduction: ``partials`` [world, ..., N] bf16 bits; sum in
    rank order in fp32 (one add per source, starting from 0), round to
    bf16. Returns bf16 bits of shape ``partials.shape[1:]``."""
    acc = np.zeros(partials.shape[1:], dtype=np.float32)
    for src in range(partials.shape[0]):
        acc = acc + from_bf16_bits(partials[src])
    return to_bf16_bits(torch.from_numpy(acc))


class PeerFabric:
    """Shared mappings standing in for symmetric peer memory: each rank owns
    ``sets`` (slab, flags) pairs in one file and maps every rank's file.

    slab(j, s)  -> uint16 [world, max_tokens, max_n]   (rank j's receive slab)
    flags(j, s) -> uint32 [world, max_units]            (rank j's flag array)
    """

    def __init__(self, rank: int, world: int, max_tokens: int, max_n: int, tile_t: int, directory: str,
                 tag: str, sets: int = 2, group=None):
        import torch.distributed as dist
        self.rank, self.world, self.sets = rank, world, sets
        self.max_tokens, self.max_n = max_tokens, max_n
        t_tiles = -(-max_tokens // tile_t)
        self.max_units = (max_n // BM) * t_tiles * (tile_t // KSLAB)
        self.slab_elems = world * max_tokens * max_n
        self.set_bytes = self.slab_elems * 2 + world * self.max_units * 4
        self.paths = [os.path.join(directory, f"{tag}.rank{j}") for j in range(world)]
        with open(self.paths[rank], "wb") as f:
            f.truncate(self.set_bytes * sets)  # zero-filled: flags start at 0
        dist.barrier(group=group)
        self._maps, self._files = [], []
        for p in self.paths:
            f = open(p, "r+b")
            self._files.append(f)
            self._maps.append(mmap.mmap(f.fileno(), self.set_bytes * sets))
        self.group = group

    def _view(self, j: int, s: int):
        base = s * self.set_bytes
        buf = self._maps[j]
        slab = np.frombuffer(buf, dtype=np.uint16, count=self.slab_elems, offset=base)
        flags = np.frombuffer(buf, dtype=np.uint32, count=self.world * self.max_units,
                              offset=base + self.slab_elems * 2)
        return (slab.reshape(self.world, self.max_tokens, self.max_n),
                flags.reshape(self.world, self.max_units))

    def slab(self, j: int, s: int) -> np.ndarray:
        return self._view(j, s)[0]

    def flags(self, j: int, s: int) -> np.ndarray:
        return self._view(j, s)[1]

    def close(self) -> None:
        import torch.distributed as dist
        dist.barrier(group=self.group)
        for m in self._maps:
            m.close()
        for f in self._files:
            f.close()
        self._maps, self._files = [], []
        dist.barrier(group=self.group)
        try:
            os.unlink(self.paths[self.rank])
        except FileNotFoundError:
            pass


class EmulatedAllReduce:
    """y = all_reduce(x @ w.T) over the ranks, by the kernel's protocol.

    ``cs`` emulates cluster split-K (counted chunk flags), ``grid`` the
    number of reducing CTAs, ``seed`` shuffles the order tiles are published
    and units reduced (a stand-in for the GPU's timing), ``budget_s`` is the
    bounded wait of step 3. ``drop`` = (tile, share) pushes this rank skips
    (a lost message); ``stall_s`` sleeps between the push and the reduce
    phase (a slow rank).
    """

    def __init__(self, fabric: PeerFabric, tile_t: int = 16, cs: int = 1, grid: int = 148,
                 budget_s: float = 2.0):
        if tile_t % KSLAB or tile_t <= 0:
            raise ValueError("tile_t is a multiple of 16")
        self.f = fabric
        self.tile_t, self.cs, self.grid, self.budget_s = tile_t, cs, grid, budget_s
        self.k = 0
        self.calls = 0

    def __call__(self, x: torch.Tensor, w: torch.Tensor, seed: int = 0, drop=(), stall_s: float = 0.0):
        f, TN, CH = self.f, self.tile_t, self.tile_t // KSLAB
        T, N = x.shape[0], w.shape[0]
        if T > f.max_tokens or N > f.max_n or N % BM:
            raise ValueError("shape outside the fabric's slab")
        s = self.k
        self.k = (self.k + 1) % f.sets
        self.calls += 1
        rng = np.random.default_rng(seed)
        part = to_bf16_bits(x.float() @ w.float().t())  # this rank's partial, bf16 bits [T, N]
        t_tiles = -(-T // TN)
        tiles = (N // BM) * t_tiles
        # steps 1-2: push every (tile, share) to every rank, then release its chunks
        pushes = [(tile, r) for tile in range(tiles) for r in range(max(1, self.cs))]
        for i in rng.permutation(len(pushes)):
            tile, r = pushes[i]
            if (tile, r) in drop:
                continue
            nt, tt = divmod(tile, t_tiles)
            t0 = tt * TN
            tv = min(TN, T - t0)
            lo, hi = share_bounds(tv, self.cs, r) if self.cs > 1 else (0, tv)
            if lo >= hi:
                continue
            rows = part[t0 + lo:t0 + hi, nt * BM:(nt + 1) * BM]
            for j in range(f.world):
                f.slab(j, s)[f.rank, t0 + lo:t0 + hi, nt * BM:(nt + 1) * BM] = rows
            for j in range(f.world):
                fl = f.flags(j, s)
                for ch in published_chunks(lo, hi):
                    fl[f.rank, tile * CH + ch] += 1
        if stall_s:
            time.sleep(stall_s)
        # step 3: reduce the owned units, CTA by CTA in a shuffled order
        status = STATUS_OK
        mine, myflags = f.slab(f.rank, s), f.flags(f.rank, s)
        out = np.zeros((T, N), dtype=np.uint16)
        units = tiles * CH
        for c in rng.permutation(min(self.grid, units)):
            for u in range(int(c), units, self.grid):
                tile, ch = divmod(u, CH)
                nt, tt = divmod(tile, t_tiles)
                t0 = tt * TN + ch * KSLAB
                if t0 >= T:
                    continue
                tv = min(TN, T - tt * TN)
                need = chunk_contributors(tv, self.cs, ch)
                deadline = time.monotonic() + self.budget_s
                while not all(myflags[src, u] >= need for src in range(f.world)):
                    if time.monotonic() > deadline:
                        status = STATUS_PEER_TIMEOUT  # as the kernel: record and go on
                        break
                    time.sleep(1e-4)
                t1 = min(t0 + KSLAB, T)
                cols = slice(nt * BM, (nt + 1) * BM)
                out[t0:t1, cols] = reduce_rank_order(mine[:, t0:t1, cols])
                myflags[:, u] = 0
        y = torch.from_numpy(out.view(np.int16).copy()).view(torch.bfloat16)
        return y, status


# ---------------------------------------------------------------------------
# The decode-size line exchange (gemm.cu: write_row's line path,
# reduce_line_row, ll_epoch / ll_finish).
#
# A call uses epoch e = state + 1 and line set e & 1. Every 4 output columns
# of a rank's bf16 partial become one 16-byte line {c0|c1, e, c2|c3, e}
# written into every rank's buffer at [set][source][token][column / 4]:
# with per-peer stores one whole line per rank; through NVLink multicast as
# two 8-byte halves, each reaching every rank's copy at once. A reader polls
# its own buffer until both halves of every source's line carry e (bounded),
# sums the sources in rank order in fp32 and rounds to bf16; no flag, fence
# or reset is involved. After the call the epoch advances (0 is skipped on
# wrap-around, so a never-written line never matches).

LINE_WORDS = 4  # u32 words per 16-byte line


class LineFabric:
    """Shared mappings standing in for the symmetric line buffers: rank j's
    buffer is ``lines(j)`` -> uint32 [2 sets, world, max_tokens, max_n / 4,
    4], zero-filled at creation (epoch 0 matches no call)."""

    def __init__(self, rank: int, world: int, max_tokens: int, max_n: int, directory: str, tag: str,
                 group=None):
        import torch.distributed as dist
        if max_n % 4:
            raise ValueError("max_n is a multiple of 4")
        self.rank, self.world, self.max_tokens, self.max_n = rank, world, max_tokens, max_n
        self.shape = (2, world, max_tokens, max_n // 4, LINE_WORDS)
        self.nbytes = int(np.prod(self.shape)) * 4
        self.paths = [os.path.join(directory, f"{tag}.lines{j}") for j in range(world)]
        with open(self.paths[rank], "wb") as f:
            f.truncate(self.nbytes)
        dist.barrier(group=group)
        self._files = [open(p, "r+b") for p in self.paths]
        self._maps = [mmap.mmap(f.fileno(), self.nbytes) for f in self._files]
        self.group = group

    def lines(self, j: int) -> np.ndarray:
        return np.frombuffer(self._maps[j], dtype=np.uint32).reshape(self.shape)

    def close(self) -> None:
        import torch.distributed as dist
        dist.barrier(group=self.group)
        for m in self._maps:
            m.close()
        for f in self._files:
            f.close()
        self._maps, self._files = [], []
        dist.barrier(group=self.group)
        try:
            os.unlink(self.paths[self.rank])
        except FileNotFoundError:
            pass


def state_after_call(e: int) -> int:
    """ll_finish: the epoch state after a call that used epoch ``e`` (the
    next call uses state + 1); 0xFFFFFFFF leaves 1, so no call ever uses
    epoch 0, the value of a never-written line."""
    return 1 if e == 0xFFFFFFFF else e


class EmulatedLineAllReduce:
    """y = all_reduce(x @ w.T) over the ranks by the line exchange.

    ``multicast``: each line leaves as two 8-byte halves, each written into
    every rank's copy before the next half (the NVLS path); otherwise each
    rank's copy receives the whole line in turn (per-peer stores).
    ``__call__`` options: ``seed`` shuffles the order lines are written;
    ``torn`` writes every line's first halves before any second half (the
    most a reader can see of 8-byte granularity); ``drop`` = token rows this
    rank does not push (a lost message); ``stall_s`` sleeps before the push
    (a slow rank). Returns (y, status) with the kernel's peer-timeout status
    when a bounded wait gave up.
    """

    def __init__(self, fabric: LineFabric, multicast: bool = False, budget_s: float = 2.0):
        self.f = fabric
        self.multicast = multicast
        self.budget_s = budget_s
        self.state = 0  # ll_state[0]: the last call's epoch

    def _push(self, e: int, set_: int, part: np.ndarray, rng, torn: bool, drop) -> None:
        f = self.f
        T, N = part.shape
        pairs = part.reshape(T, N // 4, 2, 2).astype(np.uint32)
        words = pairs[..., 0] | (pairs[..., 1] << 16)  # [T, N/4, 2]: c0|c1 and c2|c3
        rows = [t for t in range(T) if t not in drop]
        order = rng.permutation(len(rows))
        dsts = [f.lines(j)[set_, f.rank] for j in range(f.world)]
        halves = (0, 1)

        def put(t, h, dst):
            # payload word first, then its epoch word: a reader that sees
            # the epoch of a half sees that half's payload (stores become
            # visible in order)
            dst[t, :N // 4, 2 * h] = words[t, :, h]
            dst[t, :N // 4, 2 * h + 1] = e

        if torn:
            for h in halves:
                for i in order:
                    for dst in dsts:
                        put(rows[i], h, dst)
        elif self.multicast:
            for i in order:
                for h in halves:  # each 8-byte half reaches every copy before the next
                    for dst in dsts:
                        put(rows[i], h, dst)
        else:
            for dst in dsts:  # the whole line, one rank's copy after another
                for i in order:
                    for h in halves:
                        put(rows[i], h, dst)

    def __call__(self, x: torch.Tensor, w: torch.Tensor, seed: int = 0, torn: bool = False, drop=(),
                 stall_s: float = 0.0):
        f = self.f
        T, N = x.shape[0], w.shape[0]
        if T > f.max_tokens or N > f.max_n or N % 4:
            raise ValueError("shape outside the line buffers")
        e = self.state + 1  # ll_epoch
        set_ = e & 1
        rng = np.random.default_rng(seed)
        part = to_bf16_bits(x.float() @ w.float().t())  # bf16 bits [T, N]
        if stall_s:
            time.sleep(stall_s)
        self._push(e, set_, part, rng, torn, set(drop))
        # reduce_line_row: poll this rank's own copy, every source, bounded
        mine = f.lines(f.rank)[set_, :, :T, :N // 4]
        status = STATUS_OK
        deadline = time.monotonic() + self.budget_s
        while not ((mine[..., 1] == e).all() and (mine[..., 3] == e).all()):
            if time.monotonic() > deadline:
                status = STATUS_PEER_TIMEOUT  # as the kernel: record, reduce what is there
                break
            time.sleep(1e-4)
        got = mine.copy()
        lo = np.stack([got[..., 0] & 0xFFFF, got[..., 0] >> 16, got[..., 2] & 0xFFFF, got[..., 2] >> 16], -1)
        partials = lo.reshape(f.world, T, N).astype(np.uint16)
        out = reduce_rank_order(partials)
        self.state = state_after_call(e)  # ll_finish
        y = torch.from_numpy(out.view(np.int16).copy()).view(torch.bfloat16)
        return y, status
