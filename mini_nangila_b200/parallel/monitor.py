"""Host-side membership for a training loop.

Before each step every rank announces the step in the process group's
key-value store and waits (bounded) until every peer has announced it too.
A rank that leaves between steps (no kernel or collective of it in flight)
announces that instead, so the others notice before they launch an exchange
that would wait for it; a rank that crashed stays silent and the wait limit
names it.  The fused all-reduce maps every peer's symmetric
region, so teardown is ordered: the survivors unmap the leaver's region and
acknowledge in the store, and the leaver frees its own only after every
acknowledgement (or its wait limit).  No collective is involved, so nothing
hangs on the missing rank.

The reference has no failure detection; its decoders only tolerate
malformed streams.
"""
from __future__ import annotations

import time

import torch.distributed as dist

from .fused import CommError

_PREFIX = "ngl/monitor"


class RankMonitor:
    """Per-step membership handshake in the process group's store; see the module docstring."""
    def __init__(self, group=None, store=None, comms=(), timeout_s: float = 10.0):
        self.group = group
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.store = store if store is not None else (dist.distributed_c10d._get_default_store()
                                                      if dist.is_initialized() else None)
        self.comms = list(comms)
        self.timeout_s = float(timeout_s)
        self.acked: set[int] = set()

    def add_comm(self, comm) -> None:
        """Register a communicator whose symmetric region peers map."""
        self.comms.append(comm)

    def _regions(self):
        return [c.region for c in self.comms if getattr(c, "region", None) is not None]

    def check(self, step: int) -> None:
        """Before step ``step``: announce it, then wait (bounded) until every
        peer has announced it too or has left.  Raises ``CommError`` naming
        the ranks that left (after unmapping their regions and
        acknowledging) or that stayed silent past the time limit (a crash)."""
        if self.store is None or self.world == 1:
            return
        self.store.set(f"{_PREFIX}/start/{self.rank}", str(int(step)))
        pending = [r for r in range(self.world) if r != self.rank]
        left: list[int] = []
        deadline = time.monotonic() + self.timeout_s
        while pending:
            still = []
            for r in pending:
                if self.store.check([f"{_PREFIX}/left/{r}"]):
                    left.append(r)
                elif not (self.store.check([f"{_PREFIX}/start/{r}"])
                          and int(self.store.get(f"{_PREFIX}/start/{r}")) >= step):
                    still.append(r)
            pending = still
            if pending and time.monotonic() > deadline:
                break
            if pending:
                time.sleep(0.002)
        if left:
            for reg in self._regions():
                reg.unmap_peers()
            for r in left:
                if r not in self.acked:
                    self.store.add(f"{_PREFIX}/ack/{r}", 1)
                    self.acked.add(r)
        msgs = [f"rank {r} left ({self.store.get(f'{_PREFIX}/left/{r}').decode()})" for r in left]
        msgs += [f"rank {r} silent for {self.timeout_s:.0f} s before step {step}" for r in pending]
        if msgs:
            raise CommError("; ".join(msgs))

    def leave(self, reason: str = "leaving") -> bool:
        """Between steps: announce that this rank leaves, wait (bounded) until
        every peer has unmapped this rank's memory, then free it.  Returns
        whether every peer acknowledged."""
        if self.store is None or self.world == 1:
            for reg in self._regions():
                reg.free_local()
            return True
        self.store.set(f"{_PREFIX}/left/{self.rank}", reason)
        deadline = time.monotonic() + self.timeout_s
        ok = False
        while time.monotonic() < deadline:
            if int(self.store.add(f"{_PREFIX}/ack/{self.rank}", 0)) >= self.world - 1:
                ok = True
                break
            time.sleep(0.01)
        if ok:
            for reg in self._regions():
                reg.free_local()
        else:
            # A peer never acknowledged: it may still map this region, so it
            # is not freed (the process exit releases it).
            for reg in self._regions():
                reg.unmap_peers()
        return ok
