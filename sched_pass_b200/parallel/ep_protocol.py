"""CPU emulation of the expert-parallel MoE exchange (csrc/kernels/moe.cu:
``dispatch_kernel``, the expert GEMMs' wait / ``finish_gate_up`` and combine
epilogue, ``combine_norm_kernel``), run by gloo ranks over shared file
mappings that stand in for the symmetric buffers the kernels reach over
NVLink.

Per layer call, on every rank, in the kernels' order:

1. dispatch: each (token, k) assignment takes a slot on the owning rank's
   per-expert counter by an atomic add (a lock on the owner's file stands in
   for ``atomicAdd_system``); a slot at or above the capacity drops the
   assignment (its combine row is zero). A kept assignment stores the token
   row and its (source, token, k, weight) record at the owner's
   [expert][slot]. Then the source adds one to every owner's done count.
2. experts (as owner): wait, bounded, until the done count reaches the
   world size; read the row counts, clear the counters and the done count
   (``finish_gate_up``); run each expert over its rows and store each
   result, scaled by its routing weight, into the source's combine buffer at
   [token][k], counting it there.
3. combine (as source): wait, bounded, for T x K - dropped rows; sum the K
   rows in k order; clear the count.

The expert is a linear map in fp32 here (the GPU runs fp8 SwiGLU FFNs): the
emulation is about which rows go where and when, not about their
arithmetic. ``sets`` = 2 alternates two buffer sets between consecutive
calls; with one set, a source that routed nothing to a slow owner can
finish a layer, dispatch the next one and have its done count cleared by
that owner's reset of the previous layer, after which the owner's next wait
gives up (``ExpertParallel`` therefore alternates two sets).
"""
from __future__ import annotations

import fcntl
import mmap
import os
import time

import numpy as np

from .protocol import STATUS_OK, STATUS_PEER_TIMEOUT


class EpFabric:
    """Per rank and set: counters u32 [E_local], done u32, slab f32
    [E_local, cap, H], meta f32 [E_local, cap, 4] (source, token, k, weight),
    combine f32 [max_tokens, K, H], combine count u32."""

    def __init__(self, rank: int, world: int, e_local: int, cap: int, hidden: int, max_tokens: int, top_k: int,
                 directory: str, tag: str, sets: int = 2, group=None):
        import torch.distributed as dist
        self.rank, self.world, self.E_local, self.cap, self.H = rank, world, e_local, cap, hidden
        self.M, self.K, self.sets = max_tokens, top_k, sets
        self.parts = [("counter", np.uint32, (e_local,)), ("done", np.uint32, (1,)),
                      ("slab", np.float32, (e_local, cap, hidden)), ("meta", np.float32, (e_local, cap, 4)),
                      ("combine", np.float32, (max_tokens, top_k, hidden)), ("combine_cnt", np.uint32, (1,))]
        self.off, total = {}, 0
        for name, dt, shape in self.parts:
            self.off[name] = total
            total += int(np.prod(shape)) * np.dtype(dt).itemsize
        self.set_bytes = total
        self.paths = [os.path.join(directory, f"{tag}.ep{j}") for j in range(world)]
        with open(self.paths[rank], "wb") as f:
            f.truncate(self.set_bytes * sets)  # zero-filled: every count starts at 0
        dist.barrier(group=group)
        self.group = group
        self._files = [open(p, "r+b") for p in self.paths]
        self._maps = [mmap.mmap(f.fileno(), self.set_bytes * sets) for f in self._files]

    def view(self, j: int, s: int, name: str) -> np.ndarray:
        for n, dt, shape in self.parts:
            if n == name:
                return np.frombuffer(self._maps[j], dtype=dt, count=int(np.prod(shape)),
                                     offset=s * self.set_bytes + self.off[name]).reshape(shape)
        raise KeyError(name)

    def atomic_add(self, j: int, s: int, name: str, index: int, value: int = 1) -> int:
        """The old value of ``view(j, s, name)[index]``, after adding."""
        fd = self._files[j].fileno()
        fcntl.lockf(fd, fcntl.LOCK_EX)
        try:
            arr = self.view(j, s, name).reshape(-1)
            old = int(arr[index])
            arr[index] = old + value
            return old
        finally:
            fcntl.lockf(fd, fcntl.LOCK_UN)

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


class EmulatedMoEExchange:
    """One MoE layer call over the fabric: ``__call__(x, ids, wts, experts)``
    with x f32 [T, H], ids int [T, K] global expert ids, wts f32 [T, K],
    ``experts`` f32 [E_local, H, H] this rank's expert weights. Returns
    (out [T, H] = sum over kept k of w * x @ W_e^T in k order, kept mask
    [T, K], status). ``stall_s`` sleeps before the expert phase (a slow
    owner); ``budget_s`` bounds every wait."""

    def __init__(self, fabric: EpFabric, budget_s: float = 2.0):
        self.f = fabric
        self.budget_s = budget_s
        self.k = 0

    def _wait(self, arr, need: int) -> bool:
        deadline = time.monotonic() + self.budget_s
        while int(arr[0]) < need:
            if time.monotonic() > deadline:
                return False
            time.sleep(1e-4)
        return True

    def __call__(self, x: np.ndarray, ids: np.ndarray, wts: np.ndarray, experts: np.ndarray,
                 stall_s: float = 0.0):
        f = self.f
        s = self.k
        self.k = (self.k + 1) % f.sets
        T, K = ids.shape
        status = STATUS_OK
        kept = np.zeros((T, K), dtype=bool)
        mycomb = f.view(f.rank, s, "combine")
        # 1. dispatch
        for t in range(T):
            for k in range(K):
                e = int(ids[t, k])
                owner, le = divmod(e, f.E_local)
                slot = f.atomic_add(owner, s, "counter", le)
                if slot < f.cap:
                    f.view(owner, s, "slab")[le, slot] = x[t]
                    f.view(owner, s, "meta")[le, slot] = (f.rank, t, k, wts[t, k])
                    kept[t, k] = True
                else:
                    mycomb[t, k] = 0.0  # a dropped assignment adds a zero row
        for j in range(f.world):
            f.atomic_add(j, s, "done", 0)
        if stall_s:
            time.sleep(stall_s)
        # 2. experts, as owner
        done = f.view(f.rank, s, "done")
        if not self._wait(done, f.world):
            status = STATUS_PEER_TIMEOUT
        counter = f.view(f.rank, s, "counter")
        rows = np.minimum(counter.copy(), f.cap)
        counter[:] = 0  # finish_gate_up: the consumer clears the counts
        done[0] = 0
        slab, meta = f.view(f.rank, s, "slab"), f.view(f.rank, s, "meta")
        for le in range(f.E_local):
            for r in range(int(rows[le])):
                src, t, k, w = meta[le, r]
                y = (slab[le, r] @ experts[le].T) * np.float32(w)
                f.view(int(src), s, "combine")[int(t), int(k)] = y
                f.atomic_add(int(src), s, "combine_cnt", 0)
        # 3. combine, as source
        cnt = f.view(f.rank, s, "combine_cnt")
        if not self._wait(cnt, int(kept.sum())):
            status = STATUS_PEER_TIMEOUT
        out = np.zeros((T, f.H), dtype=np.float32)
        for k in range(K):
            out += mycomb[:T, k]
        cnt[0] = 0
        return out, kept, status
