"""Symmetric peer buffers over NVLink (CUDA IPC handles exchanged through
torch.distributed). ``SymmetricBuffer.ptrs[j]`` is this process's address of
rank j's buffer; kernels load/store through it directly.

``MulticastBuffer`` adds an NVLink multicast (NVLS) mapping of the same
memory, from torch's symmetric-memory allocator: ``mc`` is this process's
address of it, and a ``multimem`` store to ``mc + off`` reaches every rank's
copy at ``off`` through the switch."""
from __future__ import annotations

import torch
import torch.distributed as dist

from .._ext import ext


class SymmetricBuffer:
    def __init__(self, nbytes: int, group=None):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.nbytes = int(nbytes)
        E = ext()
        self.local, handle = E.symm_alloc(self.nbytes)
        handles = [None] * self.world
        dist.all_gather_object(handles, handle, group=group)
        self.ptrs = []
        self._opened = []
        for j, h in enumerate(handles):
            if j == self.rank:
                self.ptrs.append(self.local)
            else:
                p = E.symm_open(h)
                self._opened.append(p)
                self.ptrs.append(p)

    def close(self) -> None:
        E = ext()
        for p in self._opened:
            E.symm_close(p)
        self._opened = []
        if self.local:
            E.symm_free(self.local)
            self.local = 0

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class MulticastBuffer:
    """``nbytes`` of torch symmetric memory on ``device`` with an NVLink
    multicast mapping, zeroed on every rank before the constructor returns
    (a collective: every rank of ``group`` constructs it). ``ptrs`` and
    ``local`` as in SymmetricBuffer; ``mc``: the multicast address. Raises
    RuntimeError where the GPUs or the driver offer no multicast."""

    def __init__(self, nbytes: int, group, device):
        import torch.distributed._symmetric_memory as symm_mem
        self.group = group if group is not None else dist.group.WORLD
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.nbytes = int(nbytes)
        self._t = symm_mem.empty(self.nbytes, dtype=torch.uint8, device=device)
        self._hdl = symm_mem.rendezvous(self._t, self.group)
        if not self._hdl.multicast_ptr:  # 0 where the GPUs or the driver offer no multicast
            raise RuntimeError("no NVLink multicast for this group")
        self.mc = int(self._hdl.multicast_ptr)
        self.ptrs = [int(p) for p in self._hdl.buffer_ptrs]
        self.local = self.ptrs[self.rank]
        self._t.zero_()
        torch.cuda.synchronize(device)
        dist.barrier(group)

    def close(self) -> None:
        self._hdl = None
        self._t = None
        self.local = 0
