"""Sequence-parallel tensor parallelism: GEMM -> reduce-scatter and
all-gather -> GEMM over NVLink peer memory, with the norm between them run
once per token instead of once per rank.

Per decoder layer (T tokens, W ranks, rank r owning the token rows
[r*T/W, (r+1)*T/W)):

1. ``linear_rs`` (o_proj, down_proj): the tcgen05 GEMM with the
   ``kEpiReduceScatter`` epilogue (``csrc/kernels/gemm.cu``). Every finished
   bf16 row of the partial product goes straight from the epilogue to the
   receive slab of the rank that owns the token, followed by a row flag
   (system-scope release). Nothing is reduced in the GEMM.
2. ``reduce_norm``: ``sched_sp_reduce_norm`` (``csrc/kernels/elementwise.cu``),
   one CTA per owned row. It waits for the row's W x H/128 flags, sums the W
   partials in rank order (the fused all-reduce's exact arithmetic), adds
   the residual, applies RMSNorm, and stores the normed row into every
   rank's gather buffer (the all-gather, as peer stores), then raises the
   row's ready flag on every rank.
3. The next GEMM (QKV or gate_up) reads the local gather buffer and takes its
   ready flags as ``x_ready``: the TMA producer of each token tile waits for
   exactly that tile's rows, so the GEMM starts on the rows that have landed.

Bytes that cross NVLink per rank and projection: (W-1)/W of one [T, H]
partial for the reduce-scatter plus (W-1)/W of the normed rows for the
all-gather -- 2(W-1)/W x T x H x 2 bytes, against (W-1) x T x H x 2 for the
one-shot fused all-reduce. Residual add and RMSNorm run on T/W rows per rank
instead of T.

Buffer sets: two receive-slab sets and two gather sets alternate between
consecutive calls, as in ``parallel/fused.py``. A set's next use is
causally after every reader of its previous use (a peer needs this rank's
contribution to the intervening call first) provided every rank consumes
each gather (the next GEMM's ``x_ready`` wait, or ``wait_rows``) before its
next ``linear_rs``: with fewer tokens than ranks a rank owns no rows, and
that wait is the only thing that holds it back until its peers have read
the slab set it is about to overwrite. The model's forward always consumes
the gather; a caller that skips it can lose a row flag (the owner's wait then
ends in a peer timeout). Row flags are reset by their
reader (``reduce_norm``); the ready flags of one gather set are reset by the
next ``reduce_norm`` (which follows, in stream order, every GEMM that read
them). Per forward pass the model makes an even number of calls of each
kind, so CUDA-graph replays start on the set they were captured with.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from .. import ops
from .._ext import ext
from .symm import SymmetricBuffer


def owned_rows(rank: int, world: int, T: int) -> tuple[int, int]:
    """Token rows [lo, hi) that ``rank`` reduces and normalises (mirror of
    ``sp_row_begin`` in ``csrc/kernels/gemm_api.h``)."""
    return rank * T // world, (rank + 1) * T // world


def row_owner(t: int, world: int, T: int) -> int:
    """The rank that owns token row t (mirror of ``sp_row_owner``)."""
    return ((t + 1) * world - 1) // T


class SequenceParallel:
    def __init__(self, group, device, hidden: int, max_tokens: int = 4352):
        if hidden % 128 != 0:
            raise ValueError("hidden size must be a multiple of 128")
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.device = torch.device(device)
        self.hidden = hidden
        self.max_tokens = (max_tokens + 3) // 4 * 4  # ready flags are polled 4 at a time
        M, H, W = self.max_tokens, hidden, self.world
        self.rs = [(SymmetricBuffer(W * M * H * 2, group), SymmetricBuffer(W * (H // 128) * M * 4, group))
                   for _ in range(2)]
        self.ag = [(SymmetricBuffer(M * H * 2, group), SymmetricBuffer(M * 4, group)) for _ in range(2)]
        self.gathered = []
        for buf, _ in self.ag:
            raw = ext().symm_view(buf.local, buf.nbytes, self.device.index)
            self.gathered.append(raw.view(torch.bfloat16)[: M * H].view(M, H))
        self.k_rs = 0
        self.k_ag = 0
        self._last_rs = None
        self.calls_rs = 0
        self.calls_ag = 0

    def owned(self, T: int) -> tuple[int, int]:
        return owned_rows(self.rank, self.world, T)

    def linear_rs(self, x: torch.Tensor, w: torch.Tensor) -> None:
        """Row-parallel projection whose partial rows go to their owners."""
        T, K = x.shape
        N = w.shape[0]
        if N != self.hidden or T > self.max_tokens:
            raise ValueError(f"sequence-parallel buffers sized for N={self.hidden}, T<={self.max_tokens}")
        slab, flags = self.rs[self.k_rs]
        ws = ops.kernels._ws_for(x, N, K, 0, None)
        ext().gemm_reduce_scatter(x, w, self.rank, self.world, slab.ptrs, flags.ptrs, 0, ws.ws, ws.counters,
                                  ops.status_buffer(x.device))
        self._last_rs = self.k_rs
        self.k_rs ^= 1
        self.calls_rs += 1

    def reduce_norm(self, res: torch.Tensor, weight: torch.Tensor, eps: float, T: int,
                    delta: torch.Tensor | None = None) -> tuple[torch.Tensor, int]:
        """Reduce the owned rows of the last ``linear_rs``, residual-add
        (``res`` rows updated in place), RMSNorm, all-gather. Returns the
        gathered normed rows [T, H] (this rank's buffer) and the device
        address of their ready flags, for ``ops.linear(..., x_ready=)``."""
        if self._last_rs is None:
            raise RuntimeError("reduce_norm without a preceding linear_rs")
        slab, flags = self.rs[self._last_rs]
        self._last_rs = None
        buf, ready = self.ag[self.k_ag]
        _, other = self.ag[self.k_ag ^ 1]
        ext().sp_reduce_norm(slab.local, flags.local, res, weight, delta, buf.ptrs, ready.ptrs, other.local,
                             self.max_tokens, T, self.rank, self.world, float(eps),
                             ops.status_buffer(res.device))
        out = self.gathered[self.k_ag][:T]
        addr = ready.local
        self.k_ag ^= 1
        self.calls_ag += 1
        return out, addr

    def wait_rows(self, ready: int, T: int) -> None:
        """Order later (library) reads of gathered rows after the all-gather."""
        ext().sp_wait_rows(int(ready), int(T), ops.status_buffer(self.device))

    def close(self) -> None:
        self.gathered = []
        for a, b in self.rs + self.ag:
            a.close()
            b.close()
