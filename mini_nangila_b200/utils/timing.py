"""Device timing helpers: CUDA events on the launching stream, synchronize
on both sides, max over ranks."""
from __future__ import annotations

import time

import torch
import torch.distributed as dist


def barrier_sync(device=None) -> None:
    if dist.is_initialized():
        dist.barrier()
    if torch.cuda.is_available():
        torch.cuda.synchronize(device)


def max_over_ranks(value: float, device=None) -> float:
    if not dist.is_initialized() or dist.get_world_size() == 1:
        return float(value)
    dev = device if device is not None and torch.cuda.is_available() else ("cuda" if torch.cuda.is_available() else "cpu")
    t = torch.tensor([float(value)], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


class DeviceTimer:
    """Elapsed milliseconds between start() and stop() on the current stream."""

    def __init__(self):
        self.s = torch.cuda.Event(enable_timing=True)
        self.e = torch.cuda.Event(enable_timing=True)

    def start(self):
        self.s.record()
        return self

    def stop(self) -> float:
        self.e.record()
        self.e.synchronize()
        return self.s.elapsed_time(self.e)


class WallTimer:
    def start(self):
        self.t = time.perf_counter()
        return self

    def stop(self) -> float:
        return (time.perf_counter() - self.t) * 1000.0
