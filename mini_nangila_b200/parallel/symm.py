"""Symmetric peer memory over CUDA IPC.

Every rank allocates one region of the same size with ``cudaMalloc``, exports
an IPC handle, gathers all ranks' handles through the process group and maps
every peer's region.  Kernels then address any rank's region with a plain
device pointer: stores and loads cross NVLink / NVSwitch.  No multicast object
is created (a rank that dies while bound to one can fault its peers).
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from .._ext import cuda as _cuda


class SymmetricRegion:
    """One device allocation per rank, mapped into every peer through CUDA IPC handles."""
    def __init__(self, nbytes: int, group=None, device: torch.device | None = None):
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.device = dev
        self.nbytes = int(nbytes)
        self._region = _cuda().SymmRegion(self.nbytes, dev.index)
        handle = self._region.ipc_handle()
        if self.world > 1:
            handles = [None] * self.world
            dist.all_gather_object(handles, handle, group=group)
        else:
            handles = [handle]
        self._region.open(handles, self.rank)
        self.ptrs = list(self._region.ptrs())

    @property
    def local_ptr(self) -> int:
        return self._region.local_ptr()

    def close(self) -> None:
        """Collective: unmap peers everywhere before any rank frees its region."""
        if self._region is None:
            return
        torch.cuda.synchronize(self.device)
        self._region.close_peers()
        if self.world > 1 and dist.is_initialized():
            dist.barrier(group=self.group)
        self._region.close()
        self._region = None

    def unmap_peers(self) -> None:
        """Local, no collective: stop addressing the peers' regions (a peer
        is leaving or has left); this rank's own region stays allocated."""
        if self._region is None:
            return
        torch.cuda.synchronize(self.device)
        self._region.close_peers()

    def free_local(self) -> None:
        """Local, no collective: free this rank's region.  Only once every
        peer has unmapped it (see RankMonitor)."""
        if self._region is None:
            return
        torch.cuda.synchronize(self.device)
        self._region.close_peers()
        self._region.close()
        self._region = None
