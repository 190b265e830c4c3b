"""Row-parallel projection + all-reduce fused in one sm_100a kernel.

The GEMM's epilogue pushes each finished bf16 partial tile into every rank's
receive slab over NVLink and raises the tile's flag there; each rank then
sums the world's partials of the tiles it owns (fixed rank order: identical
results on every rank) and writes the output. Two slab sets alternate
between consecutive calls so a fast rank can run one call ahead without
overwriting data a slower rank is still reading (the next use of a set is
causally after the slow rank finished with it: the fast rank needs the slow
rank's pushes of the intervening call first).

Under CUDA graphs the sets alternate in capture order, so a replay reuses
the sequence it was captured with, and a graph that is replayed back to back
must capture an even number of calls.

Decode-sized calls (T <= ``ll_max_tokens``, ``SCHED_TP_LL_MAX``, default 32)
use the low-latency exchange instead: the partial goes out as 16-byte lines
that carry 8 bytes of bf16 and the call's epoch in each half, and the owner
of a chunk polls the lines themselves, so no system-scope fence, flag store
or flag reset sits between the GEMM and the reduction. The epoch lives in
device memory (this rank's call counter, advanced by the last CTA of each
call) and also picks which of two line-buffer sets a call uses, so graphs
replay it without host bookkeeping. The rank-order fp32 sum is the same as
the flag path's, bit for bit. The lines double the bytes on NVLink, which is
why larger calls keep the flag path.

With ``SCHED_TP_NVLS=1`` the line buffers come from torch's symmetric memory
with an NVLink multicast mapping: the epilogue writes each line once, as two
8-byte ``multimem`` stores, and the switch delivers it to every rank, instead
of one store per rank. Where the group has no multicast the IPC buffers are
used as before.
"""
from __future__ import annotations

import os

import torch

from .. import ops
from .._ext import ext
from .symm import MulticastBuffer, SymmetricBuffer

FLAG_TILES = 1 << 15  # u32 flags per source rank (covers N/128 x token tiles)


class FusedAllReduce:
    def __init__(self, group, device, max_tokens: int = 4352, max_n: int = 8192):
        import torch.distributed as dist
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.device = torch.device(device)
        self.max_tokens = max_tokens
        self.max_n = max_n
        slab = self.world * max_tokens * max_n * 2
        flags = self.world * FLAG_TILES * 4
        self.sets = [(SymmetricBuffer(slab, group), SymmetricBuffer(flags, group)) for _ in range(2)]
        self.k = 0
        self.calls = 0
        # low-latency exchange: two sets of [world][ll_max_tokens][max_n / 4] 16-byte lines
        self.ll_max_tokens = int(os.environ.get("SCHED_TP_LL_MAX", "32"))
        self.ll_calls = 0
        self._ll_last = False
        self.ll_mc = 0
        if self.ll_max_tokens > 0:
            self.ll_set_lines = self.world * self.ll_max_tokens * max_n // 4
            nbytes = 2 * self.ll_set_lines * 16
            self.ll = None
            if os.environ.get("SCHED_TP_NVLS", "0") == "1" and self.world > 1:
                try:
                    self.ll = MulticastBuffer(nbytes, group, self.device)
                    self.ll_mc = self.ll.mc
                except Exception as e:  # every rank takes the same branch: rendezvous is collective
                    print(f"[sched] NVLS line buffers unavailable ({e}); using peer stores", flush=True)
                    self.ll = None
            if self.ll is None:
                self.ll = SymmetricBuffer(nbytes, group)
            self.ll_state = torch.zeros(2, dtype=torch.int32, device=self.device)  # epoch, done
        else:
            self.ll = None

    def linear_allreduce(self, x: torch.Tensor, w: torch.Tensor, out: torch.Tensor, norm=None) -> torch.Tensor:
        """out = the all-reduced x @ w.T. ``norm = (residual, weight, eps,
        normed)`` also applies residual += out and normed = rmsnorm(residual)
        * weight inside the kernel (every rank, on its own copies)."""
        T, K = x.shape
        N = w.shape[0]
        if T > self.max_tokens or N > self.max_n:
            raise ValueError(f"fused all-reduce sized for T<={self.max_tokens}, N<={self.max_n}")
        self.calls += 1
        ws = ops.kernels._ws_for(x, N, K, 0, None)
        if norm is not None:
            res, nw, eps, normed = norm
            nargs = (res, nw, normed, ops.kernels.row_counters(x.device, T), float(eps))
        else:
            nargs = (None, None, None, None, 0.0)
        if self.ll is not None and T <= self.ll_max_tokens:
            self.ll_calls += 1
            self._ll_last = True
            ext().gemm_allreduce(x, w, out, self.rank, self.world, self.ll.ptrs, [], 0, ws.ws, ws.counters,
                                 ops.status_buffer(x.device), self.ll_state, self.ll_set_lines, *nargs, self.ll_mc)
            return out
        self._ll_last = False
        slab, flags = self.sets[self.k]
        self.k ^= 1
        ext().gemm_allreduce(x, w, out, self.rank, self.world, slab.ptrs, flags.ptrs, 0, ws.ws,
                             ws.counters, ops.status_buffer(x.device), None, 0, *nargs, 0)
        return out

    def last_slab(self, T: int, N: int) -> torch.Tensor:
        """bf16 [world, T, N]: the partials every rank pushed into this rank's
        slab in the most recent call (the inputs of its reduction)."""
        if self._ll_last:
            # line buffer of the last call's set: lines {bf16x2, epoch, bf16x2, epoch}
            e = int(self.ll_state[0].item())  # the last call's epoch
            raw = ext().symm_view(self.ll.local, self.ll.nbytes, self.device.index).view(torch.int32)
            lines = raw[(e & 1) * self.ll_set_lines * 4:][: self.world * T * N].view(-1, 4)
            payload = lines[:, [0, 2]].contiguous().view(torch.bfloat16)
            return payload.view(self.world, T, N)
        slab, _ = self.sets[self.k ^ 1]
        raw = ext().symm_view(slab.local, slab.nbytes, self.device.index)
        # the kernel packs the slab for the call's shape: [(src * T + t) * N + n]
        return raw.view(torch.bfloat16)[: self.world * T * N].view(self.world, T, N)

    def close(self):
        for a, b in self.sets:
            a.close()
            b.close()
        if self.ll is not None:
            self.ll.close()
