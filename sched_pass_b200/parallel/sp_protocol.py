"""CPU emulation of the sequence-parallel peer-buffer protocol (reduce-scatter
GEMM epilogue -> owner's reduce + residual + RMSNorm + all-gather push ->
ready-gated GEMM): the host oracle for ``parallel/sp.py`` and a test bed for
its flag logic, run by gloo ranks over shared file mappings (the image of
the symmetric buffers the kernels reach over NVLink).

It performs the steps of the kernels in their order, with the kernels' flat
layouts:

1. ``kEpiReduceScatter`` (``csrc/kernels/gemm.cu`` ``write_row`` /
   ``publish_rows_rs``): every row of this rank's bf16 partial goes to the
   slab of its owner at ``[source][t][column]``, then the owner's row flag
   ``(source * H/128 + n_tile) * T + t`` is raised;
2. ``sched_sp_reduce_norm`` (``csrc/kernels/elementwise.cu``): first the
   ready flags of the other gather set are zeroed; for each owned row a
   bounded wait on its W x H/128 flags, the partials summed in rank order
   (``protocol.reduce_rank_order``: bit for bit the kernel's sum), the
   residual added in bf16, RMSNorm, the normed row stored into every rank's
   gather buffer, the row's ready flag raised on every rank and its row
   flags cleared;
3. the consuming GEMM's producer (``wait_rows_ready``): a token tile's rows
   are read once their ready flags are raised.

The norm uses numpy fp32 arithmetic, so its output matches the GPU kernel to
a tolerance only; the reduction (``delta``) is exact. Shuffled publication
orders and a stall option stand in for the GPU's timing; ``drop`` skips
pushes (a lost message) to exercise the bounded waits.
"""
from __future__ import annotations

import mmap
import os
import time

import numpy as np
import torch

from .protocol import BM, STATUS_OK, STATUS_PEER_TIMEOUT, from_bf16_bits, reduce_rank_order, to_bf16_bits
from .sp import owned_rows, row_owner


class SpFabric:
    """Per rank and set: slab uint16 [W, M, H], row flags uint32 [W*(H/128)*M]
    (indexed with the call's T), gather uint16 [M, H], ready uint32 [M]."""

    def __init__(self, rank: int, world: int, max_tokens: int, hidden: int, directory: str, tag: str,
                 group=None):
        import torch.distributed as dist
        self.rank, self.world, self.M, self.H = rank, world, max_tokens, hidden
        self.ntl = hidden // BM
        self.n_slab = world * max_tokens * hidden
        self.n_flags = world * self.ntl * max_tokens
        self.n_gather = max_tokens * hidden
        self.set_bytes = self.n_slab * 2 + self.n_flags * 4 + self.n_gather * 2 + max_tokens * 4
        self.paths = [os.path.join(directory, f"{tag}.rank{j}") for j in range(world)]
        with open(self.paths[rank], "wb") as f:
            f.truncate(self.set_bytes * 2)  # zero-filled: every flag starts at 0
        dist.barrier(group=group)
        self.group = group
        self._files = [open(p, "r+b") for p in self.paths]
        self._maps = [mmap.mmap(f.fileno(), self.set_bytes * 2) for f in self._files]

    def _arr(self, j, s, dtype, count, offset):
        return np.frombuffer(self._maps[j], dtype=dtype, count=count, offset=s * self.set_bytes + offset)

    def slab(self, j, s):
        return self._arr(j, s, np.uint16, self.n_slab, 0).reshape(self.world, self.M, self.H)

    def row_flags(self, j, s):
        return self._arr(j, s, np.uint32, self.n_flags, self.n_slab * 2)

    def gather(self, j, s):
        return self._arr(j, s, np.uint16, self.n_gather, self.n_slab * 2 + self.n_flags * 4).reshape(self.M, self.H)

    def ready(self, j, s):
        return self._arr(j, s, np.uint32, self.M, self.n_slab * 2 + self.n_flags * 4 + self.n_gather * 2)

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


def rmsnorm_bf16(res_bits: np.ndarray, w_bits: np.ndarray, eps: float) -> np.ndarray:
    """RMSNorm of bf16 rows in fp32, rounded to bf16 (bits)."""
    v = from_bf16_bits(res_bits)
    inv = 1.0 / np.sqrt((v * v).mean(axis=-1, keepdims=True) + np.float32(eps))
    return to_bf16_bits(torch.from_numpy((v * inv * from_bf16_bits(w_bits)).astype(np.float32)))


class EmulatedSequenceParallel:
    """The three steps for one (row-parallel projection, norm) pair; two
    slab sets and two gather sets alternate as in ``SequenceParallel``."""

    def __init__(self, fabric: SpFabric, budget_s: float = 2.0, tile_t: int = 16):
        self.f = fabric
        self.budget_s = budget_s
        self.tile_t = tile_t
        self.k_rs = 0
        self.k_ag = 0
        self._last = None

    # step 1 ---------------------------------------------------------------
    def linear_rs(self, x: torch.Tensor, w: torch.Tensor, seed: int = 0, drop=()) -> np.ndarray:
        """Push this rank's partial rows to their owners. ``drop``: (t, n_tile)
        pairs not pushed. Returns the partial (bf16 bits [T, H])."""
        f = self.f
        T, H = x.shape[0], w.shape[0]
        if H != f.H or T > f.M:
            raise ValueError("shape outside the fabric")
        s = self.k_rs
        self.k_rs ^= 1
        self._last = (s, T)
        part = to_bf16_bits(x.float() @ w.float().t())
        rng = np.random.default_rng(seed)
        units = [(t, nt) for t in range(T) for nt in range(f.ntl)]
        for i in rng.permutation(len(units)):
            t, nt = units[i]
            if (t, nt) in drop:
                continue
            o = row_owner(t, f.world, T)
            f.slab(o, s)[f.rank, t, nt * BM:(nt + 1) * BM] = part[t, nt * BM:(nt + 1) * BM]
            f.row_flags(o, s)[(f.rank * f.ntl + nt) * T + t] = 1
        return part

    # step 2 ---------------------------------------------------------------
    def reduce_norm(self, res_bits: np.ndarray, w_bits: np.ndarray, eps: float, seed: int = 0,
                    stall_s: float = 0.0):
        """Reduce the owned rows, residual-add into ``res_bits`` (bf16 bits
        [T, H], owned rows updated), RMSNorm, all-gather. Returns (gather set
        index, delta bits of the owned rows [hi - lo, H], status)."""
        f = self.f
        s, T = self._last
        self._last = None
        g = self.k_ag
        self.k_ag ^= 1
        f.ready(f.rank, g ^ 1)[:] = 0  # the other set's readers are done (stream order)
        if stall_s:
            time.sleep(stall_s)
        lo, hi = owned_rows(f.rank, f.world, T)
        status = STATUS_OK
        flags = f.row_flags(f.rank, s)
        mine = f.slab(f.rank, s)
        delta = np.zeros((hi - lo, f.H), dtype=np.uint16)
        rng = np.random.default_rng(seed)
        for t in (lo + rng.permutation(hi - lo)):
            t = int(t)
            idx = [(src * f.ntl + nt) * T + t for src in range(f.world) for nt in range(f.ntl)]
            deadline = time.monotonic() + self.budget_s
            while not all(flags[i] != 0 for i in idx):
                if time.monotonic() > deadline:
                    status = STATUS_PEER_TIMEOUT  # as the kernel: record and go on
                    break
                time.sleep(1e-4)
            d = reduce_rank_order(mine[:, t:t + 1, :])[0]
            delta[t - lo] = d
            r = to_bf16_bits(torch.from_numpy(from_bf16_bits(d) + from_bf16_bits(res_bits[t])))
            res_bits[t] = r
            y = rmsnorm_bf16(r[None], w_bits, eps)[0]
            for j in range(f.world):
                f.gather(j, g)[t] = y
            for j in range(f.world):
                f.ready(j, g)[t] = 1
            for i in idx:
                flags[i] = 0
        return g, delta, status

    # step 3 ---------------------------------------------------------------
    def consume(self, g: int, T: int) -> tuple[np.ndarray, int]:
        """The consuming GEMM's view: each token tile is read once its rows'
        ready flags are raised. Returns (gathered bits [T, H], status)."""
        f = self.f
        ready = f.ready(f.rank, g)
        out = np.zeros((T, f.H), dtype=np.uint16)
        status = STATUS_OK
        for t0 in range(0, T, self.tile_t):
            t1 = min(T, t0 + self.tile_t)
            deadline = time.monotonic() + self.budget_s
            while not all(ready[t] != 0 for t in range(t0, t1)):
                if time.monotonic() > deadline:
                    status = STATUS_PEER_TIMEOUT
                    break
                time.sleep(1e-4)
            out[t0:t1] = f.gather(f.rank, g)[t0:t1]
        return out, status
