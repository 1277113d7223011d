from .fused import CommError, FusedAllReduce, autotune_twoshot, payload_bytes, topk_per_block
from .hook import HookConfig, NangilaHookState, register_nangila_hook
from .monitor import RankMonitor

__all__ = [
    "RankMonitor",
    "CommError",
    "FusedAllReduce",
    "HookConfig",
    "NangilaHookState",
    "autotune_twoshot",
    "payload_bytes",
    "register_nangila_hook",
    "topk_per_block",
]
