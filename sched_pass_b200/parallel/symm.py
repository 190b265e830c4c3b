"""Symmetric peer buffers over NVLink (CUDA IPC handles exchanged through
torch.distributed). ``SymmetricBuffer.ptrs[j]`` is this process's address of
rank j's buffer; kernels load/store through it directly."""
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
