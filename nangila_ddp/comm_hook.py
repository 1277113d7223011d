"""``nangila_ddp.comm_hook`` import path (python/nangila_ddp/comm_hook.py):
the fused sm_100a hook on CUDA models, the C++ host path on CPU."""
from mini_nangila_b200.parallel.hook import register_nangila_hook

__all__ = ["register_nangila_hook"]
