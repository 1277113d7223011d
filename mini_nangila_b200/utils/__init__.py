from .clocks import ClockSampler
from .timing import DeviceTimer, WallTimer, barrier_sync, max_over_ranks

__all__ = ["ClockSampler", "DeviceTimer", "WallTimer", "barrier_sync", "max_over_ranks"]
