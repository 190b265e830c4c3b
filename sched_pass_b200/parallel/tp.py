"""Tensor parallelism over NVLink: process group, row-parallel reductions,
vocabulary-parallel sampling.

``TensorParallel.linear_allreduce`` is the row-parallel projection
(o_proj, down_proj): every rank multiplies its K-shard and the partial sums
are added across ranks. Two implementations share the interface:

* ``fused`` (default on >= 2 GPUs): one sm_100a kernel per projection that
  runs the tcgen05 GEMM and pushes each finished bf16 partial tile to every
  peer's symmetric buffer over NVLink (peer stores), then reduces the
  peers' tiles locally after a per-chunk flag handshake (``kEpiAllReduce``
  in ``csrc/kernels/gemm.cu``; ``parallel/fused.py``);
* ``nccl``: the GEMM kernel followed by ``all_reduce`` on NCCL -- the
  baseline the fused path is measured against;
* ``sp`` (sequence parallel): the model runs its row-parallel projections as
  GEMM -> reduce-scatter, the residual add + RMSNorm on the rows each rank
  owns, and an all-gather fused into that norm that the next GEMM consumes
  tile by tile (``parallel/sp.py``); ``linear_allreduce`` itself then falls
  back to GEMM + NCCL for callers outside the decoder layer.

The fused kernel is a one-shot all-reduce: each rank pushes its whole
partial to every peer, (W - 1) x T x N x 2 bytes, where a ring or NVLS
all-reduce moves about 2 (W - 1) / W of one partial. It wins while its
lower fixed latency dominates (decode-sized T) and loses once the bytes do,
so ``fused_max_bytes`` (``SCHED_TP_FUSED_MAX_BYTES``) routes projections
whose one-shot push exceeds it to GEMM + NCCL.
"""
from __future__ import annotations

import os

import torch
import torch.distributed as dist

from .. import ops

# one-shot push bytes per rank up to which the fused kernel is used (0 = always)
DEFAULT_FUSED_MAX_BYTES = 0


class TensorParallel:
    def __init__(self, group=None, mode: str | None = None, device=None):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.device = torch.device(device) if device is not None else torch.device(
            "cuda", torch.cuda.current_device())
        self.mode = mode or os.environ.get("SCHED_TP_MODE", "fused")
        # one-shot push bytes above which the NCCL path is used (0: always fused)
        self.fused_max_bytes = int(os.environ.get("SCHED_TP_FUSED_MAX_BYTES", str(DEFAULT_FUSED_MAX_BYTES)))
        self.fused_calls = 0
        self.nccl_calls = 0
        self._fused = None
        self._sp: dict = {}  # hidden size -> SequenceParallel
        if self.mode not in ("fused", "nccl", "sp"):
            raise ValueError(f"unknown tensor-parallel mode {self.mode!r}")
        if self.mode == "fused" and self.world > 1:
            from .fused import FusedAllReduce
            self._fused = FusedAllReduce(self.group, self.device)
        # sampling exchange: two sets of [world][rows] 16-byte lines per rank
        self._sample = None
        self._sample_rows = 1024
        if self.world > 1 and os.environ.get("SCHED_TP_SAMPLE", "exchange") != "nccl":
            from .symm import SymmetricBuffer
            self._sample_set_lines = self.world * self._sample_rows
            self._sample = SymmetricBuffer(2 * self._sample_set_lines * 16, self.group)
            self._sample_state = torch.zeros(2, dtype=torch.int32, device=self.device)

    def sequence_parallel(self, hidden: int, max_tokens: int):
        """The sequence-parallel buffers of this group (``mode == "sp"``) for
        a hidden size, created on first use (collectively: every rank makes
        the same calls in the same order) and replaced by a larger set when a
        caller needs more tokens; None in the other modes."""
        if self.mode != "sp" or self.world == 1:
            return None
        sp = self._sp.get(hidden)
        if sp is None or sp.max_tokens < max_tokens:
            from .sp import SequenceParallel
            sp = self._sp[hidden] = SequenceParallel(self.group, self.device, hidden, max_tokens)
        return sp

    def use_fused(self, T: int, N: int) -> bool:
        """Whether a [T, N] row-parallel output goes through the one-shot
        fused kernel (the same answer on every rank: it depends on shapes only)."""
        if self.fused_max_bytes <= 0:
            return True
        return (self.world - 1) * T * N * 2 <= self.fused_max_bytes

    def max_over_ranks(self, value: float) -> float:
        """The maximum of a host scalar over the group (one small collective)."""
        if self.world == 1:
            return float(value)
        t = getattr(self, "_scalar", None)
        if t is None:
            t = self._scalar = torch.zeros(1, dtype=torch.float64, device=self.device)
        t.fill_(float(value))
        dist.all_reduce(t, op=dist.ReduceOp.MAX, group=self.group)
        return float(t.item())

    def linear_allreduce(self, x: torch.Tensor, w: torch.Tensor, out: torch.Tensor, norm=None) -> torch.Tensor:
        """Row-parallel projection. ``norm = (residual, weight, eps, normed)``
        also applies residual += out and normed = rmsnorm(residual) * weight:
        inside the fused kernel, or as a separate add_rmsnorm after NCCL."""
        if self.world == 1:
            if norm is not None:
                res, nw, eps, normed = norm
                ops.linear_add_rmsnorm(x, w, out, res, nw, eps, normed)
                return out
            return ops.linear(x, w, out)
        if self._fused is not None and self.use_fused(x.shape[0], w.shape[0]):
            self.fused_calls += 1
            return self._fused.linear_allreduce(x, w, out, norm=norm)
        self.nccl_calls += 1
        ops.linear(x, w, out)
        dist.all_reduce(out, group=self.group)
        if norm is not None:
            res, nw, eps, normed = norm
            ops.add_rmsnorm(out, res, nw, eps, normed)
        return out

    def sharded_argmax(self, rows: torch.Tensor, lm_head: torch.Tensor, vocab_offset: int, vocab: int,
                       out: torch.Tensor) -> torch.Tensor:
        """Greedy token over a vocabulary split across ranks: local logits, then
        one kernel that takes each row's local (max, argmax), exchanges the
        pairs with every rank over NVLink and keeps the best (lowest global id
        on ties); the same on every rank. ``SCHED_TP_SAMPLE=nccl`` (or more
        rows than the exchange holds) keeps the all-gather of the pairs."""
        S = rows.shape[0]
        logits = ops.linear(rows, lm_head)
        v_local = min(lm_head.shape[0], max(0, vocab - vocab_offset))
        if self._sample is not None and S <= self._sample_rows:
            ext = ops.kernels.ext()
            ext.argmax_exchange(logits[:, :v_local], out[:S], int(vocab_offset), self._sample.ptrs, self.rank,
                                self._sample_state, self._sample_set_lines, ops.status_buffer(rows.device))
            return out
        ids = torch.empty(S, dtype=torch.int32, device=rows.device)
        mx = torch.empty(S, dtype=torch.float32, device=rows.device)
        ops.argmax(logits[:, :v_local], ids, mx, vocab_offset)
        pair = torch.stack([mx, ids.float()], dim=0)  # exact for ids < 2^24
        allp = torch.empty(self.world, 2, S, dtype=torch.float32, device=rows.device)
        dist.all_gather_into_tensor(allp, pair, group=self.group)
        vals, gids = allp[:, 0], allp[:, 1]
        best = vals.max(dim=0).values
        cand = torch.where(vals == best[None], gids, torch.full_like(gids, float(2 ** 30)))
        out.copy_(cand.min(dim=0).values.to(torch.int32))
        return out

    def barrier(self) -> None:
        dist.barrier(group=self.group)


def init_distributed(backend: str = "nccl", timeout_s: float = 120.0):
    """Initialise torch.distributed from torchrun's environment (127.0.0.1
    rendezvous). Returns (rank, world, local_rank)."""
    import datetime
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1 and not dist.is_initialized():
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        if backend == "nccl":
            torch.cuda.set_device(local)
        dist.init_process_group(backend=backend, rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=timeout_s),
                                device_id=torch.device("cuda", local) if backend == "nccl" else None)
    return rank, world, local
