"""Peer-visible device buffers: one ``cudaMalloc`` per rank, exchanged as CUDA
IPC handles and mapped into every other rank's process (NVLink peer access)."""

from __future__ import annotations

import torch
import torch.distributed as dist

from ..ops._ext import ext


class PeerBuffer:
    """A cudaMalloc'd buffer of every rank, mapped into this process.

    ``local`` is this rank's buffer (uint8 tensor); ``ptrs`` the device array of
    every rank's base address (this rank's own entry local)."""

    def __init__(self, nbytes: int, device: torch.device, group, world: int, rank: int):
        E = ext()
        self.nbytes = int(nbytes)
        self.local, handle = E.comm_alloc(int(nbytes), device.index)
        handles = [None] * world
        dist.all_gather_object(handles, bytes(handle.tolist()), group=group)
        self.opened = []
        ptrs = []
        for r, h in enumerate(handles):
            if r == rank:
                ptrs.append(self.local.data_ptr())
            else:
                p = E.comm_ipc_open(torch.tensor(list(h), dtype=torch.uint8), device.index)
                self.opened.append(p)
                ptrs.append(p)
        self.host_ptrs = ptrs
        self.ptrs = torch.tensor(ptrs, dtype=torch.int64, device=device)

    def close(self):
        E = ext()
        for p in self.opened:
            E.comm_ipc_close(p)
        self.opened = []


__all__ = ["PeerBuffer"]
