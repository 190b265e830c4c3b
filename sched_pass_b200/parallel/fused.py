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
the sequence it was captured with. Two calls in a row on the same set are
only safe after a cross-rank synchronisation: the engine's step ends with
one (every rank waits for its step, then all-reduces the step time), and a
graph that is replayed back to back must capture an even number of calls.
"""
from __future__ import annotations

import torch

from .. import ops
from .._ext import ext
from .symm import SymmetricBuffer

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

    def linear_allreduce(self, x: torch.Tensor, w: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
        T, K = x.shape
        N = w.shape[0]
        if T > self.max_tokens or N > self.max_n:
            raise ValueError(f"fused all-reduce sized for T<={self.max_tokens}, N<={self.max_n}")
        slab, flags = self.sets[self.k]
        self.k ^= 1
        self.calls += 1
        ws = ops.kernels._ws_for(x, N, K, 0, None)
        ext().gemm_allreduce(x, w, out, self.rank, self.world, slab.ptrs, flags.ptrs, 0, ws.ws,
                             ws.counters, ops.status_buffer(x.device))
        return out

    def last_slab(self, T: int, N: int) -> torch.Tensor:
        """bf16 [world, T, N]: the partials every rank pushed into this rank's
        slab in the most recent call (the inputs of its reduction)."""
        slab, _ = self.sets[self.k ^ 1]
        raw = ext().symm_view(slab.local, slab.nbytes, self.device.index)
        # the kernel packs the slab for the call's shape: [(src * T + t) * N + n]
        return raw.view(torch.bfloat16)[: self.world * T * N].view(self.world, T, N)

    def close(self):
        for a, b in self.sets:
            a.close()
            b.close()
